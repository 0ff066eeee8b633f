"""Host logic of the PISA override and patch (CPU; no kernels run).

Mirrors the behaviours the reference pins in tests/test_pisa_patch.py:
clone-only install, explicit self-attention gate, chaining to the previous
override or the original function, the reject ladder, merged BHTD->BTC
output from the native call, and loud native failures."""
import sys
from unittest import mock

import pytest
import torch

from fakes import DummyModel, FakeCudaTensor, OtherDeviceTensor, bhtd_view
from rdna35_block_attention.pisa_patch import make_pisa_attention_override, patch_model_pisa_attention

T, D = 64, 128


def _override(previous=None, native=None):
    return make_pisa_attention_override(exact_budget=0.25, allowed_tokens=frozenset((T,)),
                                        expected_token_shape=(1, 8, 8), device_index=0,
                                        native_forward=native or mock.Mock(name="native"), verbose_fallbacks=False,
                                        previous_override=previous)


def _native_module(api=7):
    module = mock.Mock()
    module.build_info.return_value = {"api": api}
    module.capabilities.return_value = {"spatial_sparse_exact_blocks": (23,)}
    return module


def test_patch_installs_on_clone_and_chains_previous():
    previous = mock.Mock(name="previous")
    model = DummyModel({"optimized_attention_override": previous})
    with mock.patch("rdna35_block_attention.pisa_patch._device_index", return_value=(0, None)), \
            mock.patch.dict(sys.modules, {"b200_pisa": _native_module()}):
        patched, info = patch_model_pisa_attention(model, enabled=True, exact_budget=0.15625, token_policy="auto_9216",
                                                   verbose_fallbacks=False)
    assert patched is not model
    assert model.model_options["transformer_options"]["optimized_attention_override"] is previous
    assert patched.model_options["transformer_options"]["optimized_attention_override"] is not previous
    assert "generic B200 PISA" in info and "chained" in info


def test_patch_refuses_without_b200_device():
    model = DummyModel()
    with mock.patch("rdna35_block_attention.pisa_patch._device_index", return_value=(None, "sm_100 (B200) is required")):
        patched, info = patch_model_pisa_attention(model, enabled=True, exact_budget=0.15625, token_policy="auto_9216",
                                                   verbose_fallbacks=False)
    assert patched is model and "sm_100" in info


@pytest.mark.parametrize("kwargs,expected", [
    (dict(enabled=False), "disabled"),
    (dict(exact_budget=1.5), "invalid exact_budget"),
    (dict(token_policy="nope"), "unsupported token_policy"),
    (dict(start_layer=5, end_layer=2), "invalid Anima layer range"),
])
def test_patch_argument_ladder(kwargs, expected):
    args = dict(enabled=True, exact_budget=0.15625, token_policy="auto_9216", verbose_fallbacks=False)
    args.update(kwargs)
    model = DummyModel()
    patched, info = patch_model_pisa_attention(model, **args)
    assert patched is model and expected in info


def test_explicit_self_attention_marker_gates_native():
    q, k, v = bhtd_view((1, 2, T, D), value=1.0), bhtd_view((1, 2, T, D), value=2.0), bhtd_view((1, 2, T, D), value=3.0)
    previous = mock.Mock(return_value="previous")
    native = mock.Mock(return_value=torch.zeros((1, T, 2 * D), dtype=torch.bfloat16))
    override = _override(previous, native)
    assert override(mock.Mock(), q, k, v, 2, skip_reshape=True) == "previous"
    assert override(mock.Mock(), q, k, v, 2, skip_reshape=True, is_self_attention=False) == "previous"
    override(mock.Mock(), q, k, v, 2, skip_reshape=True, is_self_attention=True, is_initial_transformer_block=False,
             attention_token_shape=(1, 8, 8))
    assert previous.call_count == 2
    native.assert_called_once()


def test_unsupported_calls_reach_previous_or_original():
    q = torch.zeros((1, 2, 64, D), dtype=torch.bfloat16)
    previous, original = mock.Mock(return_value="previous"), mock.Mock(return_value="original")
    assert _override(previous)(original, q, q, q, 2, skip_reshape=True, is_self_attention=False) == "previous"
    original.assert_not_called()
    assert _override()(original, q, q, q, 2, skip_reshape=True, is_self_attention=False) == "original"
    original.assert_called_once()


CASES = [
    ("mask", lambda q, k, v: ((q, k, v), {"mask": object()})),
    ("reshape_required", lambda q, k, v: ((q, k, v), {"skip_reshape": False})),
    ("unmerged_output", lambda q, k, v: ((q, k, v), {"skip_output_reshape": True})),
    ("mismatched_shape", lambda q, k, v: ((q, bhtd_view((1, 2, T - 1, D)), v), {})),
    ("heads", lambda q, k, v: ((q, k, v), {"heads": 1})),
    ("head_dim", lambda q, k, v: ((bhtd_view((1, 2, T, 64)),) * 3, {})),
    ("dtype", lambda q, k, v: ((bhtd_view((1, 2, T, D), dtype=torch.float16),) * 3, {})),
    ("mixed_dtype", lambda q, k, v: ((q, bhtd_view((1, 2, T, D), dtype=torch.float16), v), {})),
    ("other_device", lambda q, k, v: ((q, bhtd_view((1, 2, T, D), cls=OtherDeviceTensor), v), {})),
    ("requires_grad", lambda q, k, v: ((bhtd_view((1, 2, T, D), requires_grad=True), k, v), {})),
    ("token_count", lambda q, k, v: ((bhtd_view((1, 2, 128, D)),) * 3, {})),
    ("fp32_precision", lambda q, k, v: ((q, k, v), {"attn_precision": torch.float32})),
    ("gqa", lambda q, k, v: ((q, k, v), {"enable_gqa": True})),
    ("contiguous_bhtd", lambda q, k, v: (tuple(FakeCudaTensor(x.contiguous()) for x in (q, k, v)), {})),
    ("token_shape", lambda q, k, v: ((q, k, v), {"attention_token_shape": (1, 4, 16)})),
    ("initial_block", lambda q, k, v: ((q, k, v), {"is_initial_transformer_block": True})),
]


@pytest.mark.parametrize("name,make", CASES, ids=[c[0] for c in CASES])
def test_ineligible_calls_never_reach_native(name, make):
    q, k, v = (bhtd_view((1, 2, T, D), value=x) for x in (1.0, 2.0, 3.0))
    tensors, kwargs = make(q, k, v)
    heads = kwargs.pop("heads", 2)
    call = dict(skip_reshape=True, is_self_attention=True, is_initial_transformer_block=False,
                attention_token_shape=(1, 8, 8))
    call.update(kwargs)
    previous, native = mock.Mock(return_value="previous"), mock.Mock()
    assert _override(previous, native)(mock.Mock(), *tensors, heads, **call) == "previous"
    previous.assert_called_once()
    native.assert_not_called()


def test_cpu_tensors_fall_back():
    cpu = torch.zeros((1, 2, T, D), dtype=torch.bfloat16)
    previous, native = mock.Mock(return_value="previous"), mock.Mock()
    assert _override(previous, native)(mock.Mock(), cpu, cpu, cpu, 2, skip_reshape=True, is_self_attention=True,
                                       is_initial_transformer_block=False) == "previous"
    native.assert_not_called()


def test_eligible_call_forwards_views_and_returns_merged_output():
    q, k, v = (bhtd_view((2, 2, T, D), value=x) for x in (1.0, 2.0, 3.0))
    merged = torch.zeros((2, T, 2 * D), dtype=torch.bfloat16)
    native = mock.Mock(return_value=merged)
    out = _override(native=native)(mock.Mock(), q, k, v, 2, skip_reshape=True, is_self_attention=True,
                                   is_initial_transformer_block=False, attention_token_shape=(1, 8, 8))
    args = native.call_args.args
    assert args[0] is q and args[1] is k and args[2] is v  # no layout copy in Python
    assert args[3] == 1  # ceil(0.25 * 1 block)
    assert out is merged


def test_native_failure_is_loud():
    q = bhtd_view((1, 2, T, D), value=1.0)
    previous, original = mock.Mock(return_value="previous"), mock.Mock(return_value="original")
    override = _override(previous, mock.Mock(side_effect=RuntimeError("native failure")))
    with pytest.raises(RuntimeError, match="native failure"):
        override(original, q, q, q, 2, skip_reshape=True, is_self_attention=True, is_initial_transformer_block=False,
                 attention_token_shape=(1, 8, 8))
    previous.assert_not_called()
    original.assert_not_called()
