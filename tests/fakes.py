"""CPU stand-ins for the host-logic tests: tensors that report a CUDA
device while living on the CPU, and a ComfyUI ModelPatcher double."""
import torch


class FakeCudaTensor(torch.Tensor):
    device_index = 0

    @staticmethod
    def __new__(cls, tensor):
        return torch.Tensor._make_subclass(cls, tensor, tensor.requires_grad)

    @property
    def device(self):
        return torch.device("cuda", self.device_index)

    @property
    def is_cuda(self):
        return True


class OtherDeviceTensor(FakeCudaTensor):
    device_index = 1


def bhtd_view(shape, *, value=0.0, dtype=torch.bfloat16, requires_grad=False, cls=FakeCudaTensor):
    """[B,H,T,D] view over contiguous [B,T,H,D] storage (the ComfyUI skip_reshape layout)."""
    b, h, t, d = shape
    storage = torch.full((b, t, h, d), value, dtype=dtype, requires_grad=requires_grad)
    return cls(storage.permute(0, 2, 1, 3))


class DummyModel:
    """ModelPatcher double with clone() and model_options only."""

    def __init__(self, transformer_options=None):
        self.model_options = {"transformer_options": dict(transformer_options or {})}

    def clone(self):
        return DummyModel(self.model_options["transformer_options"])
