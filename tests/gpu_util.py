"""Helpers shared by the GPU parity tests."""
import torch

DEV = torch.device("cuda", 0) if torch.cuda.is_available() else None


def to_dev_bhtd(x_bhtd: torch.Tensor) -> torch.Tensor:
    """Move a BHTD view of BTHD storage to the GPU keeping that storage layout."""
    return x_bhtd.permute(0, 2, 1, 3).contiguous().to(DEV).permute(0, 2, 1, 3)
