"""Host logic of the Anima attn_op patch, MiniMax-H3 override, fixed-block
dispatch / ComfyUI patch and runtime accounting (CPU; kernels mocked or
not reached).  Mirrors the reference's tests/test_anima_pisa_integration.py,
test_minimax_h3_gfx1151_attention.py, test_dispatch_fallbacks.py and
test_pisa_runtime*.py behaviours."""
from types import SimpleNamespace
from unittest import mock

import pytest
import torch

from fakes import DummyModel, FakeCudaTensor
from rdna35_block_attention import minimax_h3_gfx1151_attention as h3
from rdna35_block_attention.anima_pisa_integration import (ANIMA_PISA_HEAD_DIM, ANIMA_PISA_HEADS, ANIMA_PISA_TOKENS,
                                                            install_anima_pisa_attention, make_anima_pisa_attn_op)
from rdna35_block_attention.comfy_patch import patch_model_attention
from rdna35_block_attention.dispatch import fixed_block_attention
from rdna35_block_attention.pisa_runtime import PISARuntimeState
from rdna35_block_attention.reference import fixed_block_attention_ref


# ---------------------------------------------------------------- Anima attn_op
def _anima_qkv(tokens=ANIMA_PISA_TOKENS):
    return tuple(FakeCudaTensor(torch.zeros((1, tokens, ANIMA_PISA_HEADS, ANIMA_PISA_HEAD_DIM), dtype=torch.bfloat16))
                 for _ in range(3))


class Patcher:
    def __init__(self):
        attn = SimpleNamespace(n_heads=16, head_dim=128, attn_op=lambda *a, **k: "original")
        self.diffusion_model = SimpleNamespace(blocks=[SimpleNamespace(self_attn=attn) for _ in range(28)])
        self.object_patches = {}

    def get_model_object(self, name):
        return self.diffusion_model

    def add_object_patch(self, name, obj):
        self.object_patches[name] = obj


def test_anima_op_calls_native_on_bhtd_views():
    q, k, v = _anima_qkv()
    out = torch.zeros((1, ANIMA_PISA_TOKENS, 2048), dtype=torch.bfloat16)
    native, original = mock.Mock(return_value=out), mock.Mock()
    state = PISARuntimeState(armed=True)
    op = make_anima_pisa_attn_op(original, native_forward=native, exact_blocks=23, device_index=0, layer_index=4,
                                 runtime_state=state)
    assert op(q, k, v).shape == (1, ANIMA_PISA_TOKENS, 2048)
    original.assert_not_called()
    assert native.call_args.kwargs["exact_blocks"] == 23
    assert native.call_args.args[0].shape == (1, 16, ANIMA_PISA_TOKENS, 128)
    assert native.call_args.args[0].stride() == (ANIMA_PISA_TOKENS * 2048, 128, 2048, 1)
    assert state.per_layer_hits == {4: 1}


def test_anima_other_profile_goes_to_original():
    q, k, v = _anima_qkv(tokens=64)
    original = mock.Mock(return_value="fallback")
    state = PISARuntimeState(armed=True)
    op = make_anima_pisa_attn_op(original, native_forward=mock.Mock(), exact_blocks=23, device_index=0, layer_index=4,
                                 runtime_state=state)
    assert op(q, k, v) == "fallback"
    original.assert_called_once_with(q, k, v, transformer_options=None)
    assert state.fallback_reasons["shape_(64, 16, 128)_is_not_t9216_h16_d128"] == 1


def test_anima_native_failure_is_loud():
    q, k, v = _anima_qkv()
    state = PISARuntimeState(armed=True)
    op = make_anima_pisa_attn_op(mock.Mock(), native_forward=mock.Mock(side_effect=ValueError("boom")), exact_blocks=23,
                                 device_index=0, layer_index=4, runtime_state=state)
    with pytest.raises(RuntimeError, match="eligible Anima"):
        op(q, k, v)
    assert state.failed


def test_anima_installs_requested_layers():
    patcher = Patcher()
    assert install_anima_pisa_attention(patcher, native_forward=mock.Mock(), exact_blocks=23, device_index=0,
                                        first_layer=8, last_layer=19) == 12
    assert "diffusion_model.blocks.7.self_attn.attn_op" not in patcher.object_patches
    assert "diffusion_model.blocks.8.self_attn.attn_op" in patcher.object_patches
    assert "diffusion_model.blocks.19.self_attn.attn_op" in patcher.object_patches
    assert "diffusion_model.blocks.20.self_attn.attn_op" not in patcher.object_patches


# ---------------------------------------------------------------- MiniMax-H3
def _views(tokens, heads=1, d=1):
    qkv = torch.arange(tokens * 3 * heads * d, dtype=torch.float32).reshape(1, tokens, 3, heads, d)
    return tuple(qkv[:, :, i].permute(0, 2, 1, 3) for i in range(3))


def test_h3_pack_profiles_keep_values_in_one_allocation():
    q, k, v = _views(9170)
    pq, pk, pv, profile = h3.pack_minimax_h3_qkv(q, k, v)
    assert profile == "kv" and pq is q
    assert pk.is_contiguous() and torch.equal(pk, k) and torch.equal(pv, v) and pk._base is pv._base
    q, k, v = _views(12000)
    pq, pk, pv, profile = h3.pack_minimax_h3_qkv(q, k, v)
    assert profile == "qkv" and all(torch.equal(a, b) for a, b in ((pq, q), (pk, k), (pv, v)))
    assert pq._base is pk._base is pv._base


def test_h3_reject_ladder():
    q = torch.randn(1, 56, 8, 128, dtype=torch.bfloat16)
    assert h3._reject_reason(q, q, q, 56, None, True, False, 0, {}) == "tokens_below_4608"
    big = torch.empty(1, 56, 16501, 128, dtype=torch.bfloat16, device="meta")
    assert h3._reject_reason(big, big, big, 56, None, True, False, 0, {}) == "tokens_above_16500"
    assert h3._reject_reason(q, q, q, 56, object(), True, False, 0, {}) == "attention_mask_is_not_supported"
    assert h3._reject_reason(q, q, q, 56, None, False, False, 0, {}) == "minimax_h3_merged_output_contract_is_required"
    assert h3._reject_reason(q, q, q, 56, None, True, False, 0, {"is_causal": True}) == "causal_attention_is_not_supported"


def test_h3_pack_mode_chains_previous_with_packed_tensors():
    q = torch.randn(1, 2, 3, 4)
    calls = []

    def previous(original, pq, pk, pv, heads, **kwargs):
        calls.append((heads, kwargs))
        return "previous"

    override = h3.make_minimax_h3_gfx1151_attention_override(device_index=0, verbose_fallbacks=False,
                                                             previous_override=previous, use_b200_attention=False)
    with mock.patch.object(h3, "_reject_reason", return_value=None):
        assert override(lambda *a, **k: "original", q, q.clone(), q.clone(), 2, skip_reshape=True) == "previous"
    assert calls[0][0] == 2 and calls[0][1]["skip_reshape"]


def test_h3_native_mode_runs_native_attention():
    q = torch.randn(1, 2, 3, 4)
    override = h3.make_minimax_h3_gfx1151_attention_override(device_index=0, verbose_fallbacks=False,
                                                             previous_override=None)
    with mock.patch.object(h3, "_reject_reason", return_value=None), \
            mock.patch.object(h3, "minimax_h3_attention", return_value="native") as native:
        assert override(lambda *a, **k: "original", q, q, q, 2, skip_reshape=True, scale=0.5) == "native"
    assert native.call_args.kwargs["scale"] == 0.5


def test_h3_patch_is_model_local_and_respects_container_override():
    model = DummyModel()
    patched, info = h3.patch_minimax_h3_gfx1151_attention(model, enabled=True, verbose_fallbacks=False)
    assert patched is model and "not found" in info


# ---------------------------------------------------------------- fixed block
def test_dispatch_reasons_on_cpu():
    q = torch.randn(1, 1, 64, 32, dtype=torch.float16)
    out, info = fixed_block_attention(q, q, q, layout="bhtd", return_diagnostics=True)
    assert out.shape == q.shape and info["backend"] == "reference" and "not_cuda" in info["fallback_reason"]
    _, info = fixed_block_attention(q, q, q, block_size=32, layout="bhtd", return_diagnostics=True)
    assert "unsupported_block_size_32" in info["fallback_reason"]
    # float and bool masks run natively on a GPU; on the CPU the device decides
    _, info = fixed_block_attention(q, q, q, layout="bhtd", mask=torch.zeros(64, 64), return_diagnostics=True)
    assert "not_cuda" in info["fallback_reason"]
    # masks of other dtypes keep the reference's reason
    _, info = fixed_block_attention(q, q, q, layout="bhtd", mask=torch.zeros(64, 64, dtype=torch.int32),
                                    return_diagnostics=True)
    assert "arbitrary_mask" in info["fallback_reason"]
    qg = torch.randn(1, 1, 64, 32, dtype=torch.float16, requires_grad=True)
    _, info = fixed_block_attention(qg, qg, qg, layout="bhtd", return_diagnostics=True)
    assert "requires_grad" in info["fallback_reason"]
    q160 = torch.randn(1, 1, 64, 160, dtype=torch.float16)
    _, info = fixed_block_attention(q160, q160, q160, layout="bhtd", return_diagnostics=True)
    assert "unsupported_head_dim_160" in info["fallback_reason"]


def test_dispatch_reference_mode_matches_loop():
    q, k, v = (torch.randn(2, 130, 3 * 16) for _ in range(3))
    out = fixed_block_attention(q, k, v, layout="bthd", heads=3, mode="reference")
    torch.testing.assert_close(out, fixed_block_attention_ref(q, k, v, layout="bthd", heads=3))


def test_fixed_block_patch_is_model_local_and_exact_only_passes_unmarked_calls():
    model = DummyModel()
    patched, info = patch_model_attention(model, enabled=True, mode="auto", semantic_mode="exact_only", block_size=64,
                                          causal=False, verbose_fallbacks=False)
    assert patched is not model and "exact_only" in info
    assert "optimized_attention_override" not in model.model_options["transformer_options"]
    override = patched.model_options["transformer_options"]["optimized_attention_override"]
    q = torch.randn(1, 64, 32)
    assert override(lambda *a, **k: "original", q, q, q, 1) == "original"
    marked = override(lambda *a, **k: "original", q, q, q, 1,
                      transformer_options={"rdna35_attention_semantics": "fixed_block_diagonal"})
    torch.testing.assert_close(marked, fixed_block_attention_ref(q, q, q, layout="bthd", heads=1))


# ---------------------------------------------------------------- runtime accounting
def test_runtime_verify_and_report():
    state = PISARuntimeState(armed=True, expected_layers=(20, 21))
    for layer in (20, 21, 20, 21):
        state.record(layer=layer, is_self_attention=True, shape=(1, 16, 9216, 128))
    state.record(is_self_attention=False, fallback_reason="cross")
    assert state.verify(2)
    report = state.report()
    assert "hits=4/4" in report and "fallbacks=cross:1" in report and "self=4 cross=1" in report
    state.record(layer=22)
    assert not state.verify(2) and state.failed


def test_runtime_error_marks_failed_and_reset_clears():
    state = PISARuntimeState(armed=True)
    state.record(error=RuntimeError("x"))
    assert state.failed and state.first_error == "x"
    state.reset(armed=False)
    assert not state.failed and not state.armed and state.first_error is None
    with pytest.raises(ValueError):
        PISARuntimeState.expected_calls(-1)
