"""ComfyUI nodes (same class names, widgets and return types as the
reference's nodes.py:30-609): three patch nodes, benchmark nodes measured
with CUDA-event medians / alternating A-B sampling, the PISA runtime report
and a diagnostics node."""
from __future__ import annotations

import statistics
import time
from typing import Any

import torch

from .rdna35_block_attention.anima_pisa_integration import ANIMA_PISA_FIRST_LAYER, ANIMA_PISA_LAST_LAYER
from .rdna35_block_attention.comfy_patch import patch_model_attention
from .rdna35_block_attention.device import explain_dispatch
from .rdna35_block_attention.dispatch import fixed_block_attention
from .rdna35_block_attention.full_attention import full_attention_b200
from .rdna35_block_attention.minimax_h3_gfx1151_attention import (minimax_h3_attention, minimax_h3_pack_profile,
                                                                  pack_minimax_h3_qkv,
                                                                  patch_minimax_h3_gfx1151_attention)
from .rdna35_block_attention.pisa_attention import pisa_attention
from .rdna35_block_attention.pisa_patch import patch_model_pisa_attention
from .rdna35_block_attention.pisa_runtime import PISA_RUNTIME_ATTACHMENT
from .rdna35_block_attention.reference import (fixed_block_attention_ref, fixed_block_attention_sdpa,
                                               full_attention_sdpa_bhtd)


def _sync(device: torch.device) -> None:
    if device.type == "cuda":
        torch.cuda.synchronize(device)


def _median_ms(fn, device: torch.device, iterations: int = 20, warmup: int = 5) -> float:
    for _ in range(warmup):
        fn()
    _sync(device)
    if device.type == "cuda":
        events = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(iterations)]
        for start, end in events:
            start.record()
            fn()
            end.record()
        torch.cuda.synchronize(device)
        return float(statistics.median(s.elapsed_time(e) for s, e in events))
    samples = []
    for _ in range(iterations):
        t0 = time.perf_counter()
        fn()
        samples.append((time.perf_counter() - t0) * 1e3)
    return float(statistics.median(samples))


def _alternating_medians_ms(first_fn, second_fn, device: torch.device, iterations: int, warmup: int):
    for _ in range(warmup):
        first_fn()
        second_fn()
    _sync(device)
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(iterations)]
    for a0, a1, b0, b1 in ev:
        a0.record()
        first_fn()
        a1.record()
        b0.record()
        second_fn()
        b1.record()
    torch.cuda.synchronize(device)
    return (float(statistics.median(a0.elapsed_time(a1) for a0, a1, _, _ in ev)),
            float(statistics.median(b0.elapsed_time(b1) for _, _, b0, b1 in ev)))


class RDNA35BlockAttentionDiagnostics:
    @classmethod
    def INPUT_TYPES(cls):
        return {"required": {}}

    RETURN_TYPES = ("STRING",)
    RETURN_NAMES = ("diagnostics",)
    FUNCTION = "run"
    CATEGORY = "RDNA35/Fixed Block Attention"
    OUTPUT_NODE = True

    def run(self):
        return (explain_dispatch(),)


class RDNA35PatchModelAttention:
    @classmethod
    def INPUT_TYPES(cls):
        return {"required": {
            "model": ("MODEL",),
            "enabled": ("BOOLEAN", {"default": True}),
            "mode": (["auto", "reference", "triton"], {"default": "auto"}),
            "semantic_mode": (["exact_only", "experimental_force_block_local"], {"default": "exact_only"}),
            "block_size": ("INT", {"default": 64, "min": 64, "max": 64, "step": 64}),
            "causal": ("BOOLEAN", {"default": False}),
            "verbose_fallbacks": ("BOOLEAN", {"default": False}),
        }}

    RETURN_TYPES = ("MODEL", "STRING")
    RETURN_NAMES = ("model", "info")
    FUNCTION = "patch"
    CATEGORY = "RDNA35/Fixed Block Attention"
    EXPERIMENTAL = True

    def patch(self, model, enabled, mode, semantic_mode, block_size, causal, verbose_fallbacks):
        return patch_model_attention(model, enabled=enabled, mode=mode, semantic_mode=semantic_mode,
                                     block_size=block_size, causal=causal, verbose_fallbacks=verbose_fallbacks)


class RDNA35PatchAnimaPISAAttention:
    @classmethod
    def INPUT_TYPES(cls):
        return {"required": {"model": ("MODEL",), "enabled": ("BOOLEAN", {"default": True}),
                             "verbose_fallbacks": ("BOOLEAN", {"default": False})},
                "optional": {"first_pisa_layer": ("INT", {"default": ANIMA_PISA_FIRST_LAYER, "min": 0, "max": 27}),
                             "last_pisa_layer": ("INT", {"default": ANIMA_PISA_LAST_LAYER, "min": 0, "max": 27})}}

    RETURN_TYPES = ("MODEL", "STRING")
    RETURN_NAMES = ("model", "info")
    FUNCTION = "patch"
    CATEGORY = "RDNA35/Attention Research"
    EXPERIMENTAL = True

    def patch(self, model, enabled, verbose_fallbacks, first_pisa_layer=ANIMA_PISA_FIRST_LAYER,
              last_pisa_layer=ANIMA_PISA_LAST_LAYER):
        return patch_model_pisa_attention(model, enabled=enabled, exact_budget=0.15625,
                                          token_policy="anima_1536_spatial", start_layer=first_pisa_layer,
                                          end_layer=last_pisa_layer, verbose_fallbacks=verbose_fallbacks)


class RDNA35PatchMiniMaxH3GFX1151Attention:
    @classmethod
    def INPUT_TYPES(cls):
        return {"required": {"model": ("MODEL",), "enabled": ("BOOLEAN", {"default": True}),
                             "verbose_fallbacks": ("BOOLEAN", {"default": False})}}

    RETURN_TYPES = ("MODEL", "STRING")
    RETURN_NAMES = ("model", "info")
    FUNCTION = "patch"
    CATEGORY = "RDNA35/Attention Research"
    EXPERIMENTAL = True

    def patch(self, model, enabled, verbose_fallbacks):
        return patch_minimax_h3_gfx1151_attention(model, enabled=enabled, verbose_fallbacks=verbose_fallbacks)


class RDNA35FixedBlockAttentionBenchmark:
    @classmethod
    def INPUT_TYPES(cls):
        return {"required": {
            "batch": ("INT", {"default": 1, "min": 1, "max": 8}),
            "heads": ("INT", {"default": 4, "min": 1, "max": 32}),
            "tokens": ("INT", {"default": 128, "min": 1, "max": 8192, "step": 64}),
            "head_dim": ("INT", {"default": 64, "min": 32, "max": 128, "step": 32}),
            "dtype": (["float16", "bfloat16"], {"default": "float16"}),
            "mode": (["auto", "triton", "reference"], {"default": "auto"}),
            "causal": ("BOOLEAN", {"default": False}),
        }}

    RETURN_TYPES = ("STRING",)
    RETURN_NAMES = ("benchmark",)
    FUNCTION = "run"
    CATEGORY = "RDNA35/Fixed Block Attention"
    OUTPUT_NODE = True

    def run(self, batch, heads, tokens, head_dim, dtype, mode, causal):
        device = torch.device("cuda") if torch.cuda.is_available() else torch.device("cpu")
        dt = torch.float16 if dtype == "float16" else torch.bfloat16
        q = torch.randn(batch, heads, tokens, head_dim, device=device, dtype=dt)
        k, v = torch.randn_like(q), torch.randn_like(q)
        ref = fixed_block_attention_ref(q, k, v, causal=causal, layout="bhtd")
        out, info = fixed_block_attention(q, k, v, causal=causal, layout="bhtd", mode=mode, return_diagnostics=True)
        ref_ms = _median_ms(lambda: fixed_block_attention_ref(q, k, v, causal=causal, layout="bhtd"), device)
        sdpa_ms = _median_ms(lambda: fixed_block_attention_sdpa(q, k, v, causal=causal, layout="bhtd"), device)
        full_ms = _median_ms(lambda: full_attention_sdpa_bhtd(q, k, v, causal=causal), device)
        lines = ["RDNA35 Fixed Block Attention Benchmark (B200)",
                 f"shape: B={batch} H={heads} T={tokens} D={head_dim} dtype={dt} causal={causal}",
                 f"reference median: {ref_ms:.3f} ms", f"PyTorch SDPA block-mask median: {sdpa_ms:.3f} ms",
                 f"PyTorch SDPA full-attention median: {full_ms:.3f} ms",
                 f"dispatch backend: {info.get('backend')}", f"fallback reason: {info.get('fallback_reason')}",
                 f"max abs error vs reference: {(out.float() - ref.float()).abs().max().item():.6g}"]
        if info.get("backend") == "b200":
            ms = _median_ms(lambda: fixed_block_attention(q, k, v, causal=causal, layout="bhtd", mode="b200"), device)
            lines += [f"b200 median: {ms:.3f} ms", f"measured speedup vs reference: {ref_ms / ms:.3f}x",
                      f"measured speedup vs PyTorch SDPA block-mask: {sdpa_ms / ms:.3f}x"]
        else:
            lines.append("measured speedup: unavailable because optimized path did not run")
        return ("\n".join(lines),)


class RDNA35FullAttentionBenchmark:
    @classmethod
    def INPUT_TYPES(cls):
        return {"required": {
            "batch": ("INT", {"default": 1, "min": 1, "max": 4}),
            "heads": ("INT", {"default": 16, "min": 1, "max": 40}),
            "query_tokens": ("INT", {"default": 4096, "min": 64, "max": 9216, "step": 64}),
            "key_tokens": ("INT", {"default": 4096, "min": 64, "max": 9216, "step": 64}),
            "head_dim": ([64, 128], {"default": 128}),
            "dtype": (["float16", "bfloat16"], {"default": "bfloat16"}),
        }}

    RETURN_TYPES = ("STRING",)
    RETURN_NAMES = ("benchmark",)
    FUNCTION = "run"
    CATEGORY = "RDNA35/Attention Research"
    OUTPUT_NODE = True
    EXPERIMENTAL = True

    def run(self, batch, heads, query_tokens, key_tokens, head_dim, dtype):
        device = torch.device("cuda")
        dt = torch.float16 if dtype == "float16" else torch.bfloat16
        q = torch.randn(batch, heads, query_tokens, head_dim, device=device, dtype=dt)
        k = torch.randn(batch, heads, key_tokens, head_dim, device=device, dtype=dt)
        v = torch.randn_like(k)
        qf, kf, vf = (x.flatten(0, 1).contiguous() for x in (q, k, v))
        ref = torch.nn.functional.scaled_dot_product_attention(q, k, v)
        out, info = full_attention_b200(qf, kf, vf, return_diagnostics=True)
        sdpa_ms = _median_ms(lambda: torch.nn.functional.scaled_dot_product_attention(q, k, v), device)
        ms = _median_ms(lambda: full_attention_b200(qf, kf, vf), device)
        return ("\n".join([
            "RDNA35 Exact Full Attention Benchmark (B200)",
            f"shape: B={batch} H={heads} Q={query_tokens} K={key_tokens} D={head_dim} dtype={dt}",
            f"PyTorch SDPA median: {sdpa_ms:.3f} ms", f"B200 kernel median: {ms:.3f} ms",
            f"B200/SDPA ratio: {ms / sdpa_ms:.3f}x",
            f"max abs error: {(out.unflatten(0, (batch, heads)).float() - ref.float()).abs().max().item():.6g}",
            f"kernel config: {info.get('config')}"]),)


class RDNA35MiniMaxH3GFX1151AttentionBenchmark:
    @classmethod
    def INPUT_TYPES(cls):
        return {"required": {"tokens": ("INT", {"default": 9170, "min": 4608, "max": 16500, "step": 1})}}

    RETURN_TYPES = ("STRING",)
    RETURN_NAMES = ("benchmark",)
    FUNCTION = "run"
    CATEGORY = "RDNA35/Attention Research"
    OUTPUT_NODE = True
    EXPERIMENTAL = True

    def run(self, tokens):
        device = torch.device("cuda")
        qkv = torch.randn(1, tokens, 3, 56, 128, device=device, dtype=torch.bfloat16)
        q = qkv[:, :, 0].permute(0, 2, 1, 3)
        k = qkv[:, :, 1].permute(0, 2, 1, 3)
        v = qkv[:, :, 2].clone().permute(0, 2, 1, 3)

        def existing():
            return torch.nn.functional.scaled_dot_product_attention(q, k, v).transpose(1, 2).contiguous()

        def native():
            return minimax_h3_attention(q, k, v)

        a, b = existing(), native()
        if not torch.isfinite(b).all() or not torch.allclose(b.float(), a.flatten(2).float(), atol=5e-2, rtol=5e-2):
            raise RuntimeError("B200 H3 attention failed the BF16 correctness check")
        existing_ms, native_ms = _alternating_medians_ms(existing, native, device, iterations=5, warmup=2)
        return ("\n".join([
            "RDNA35 MiniMax-H3 Attention Benchmark (B200)",
            f"shape: B=1 H=56 T={tokens} D=128 dtype=bfloat16",
            f"packing profile of the reference path: {minimax_h3_pack_profile(tokens).upper()}",
            f"existing strided SDPA median: {existing_ms:.3f} ms", f"B200 native median: {native_ms:.3f} ms",
            f"measured speedup: {existing_ms / native_ms:.3f}x",
            f"max abs error: {(b.float() - a.flatten(2).float()).abs().max().item():.6g}"]),)


class RDNA35PISAAttentionBenchmark:
    @classmethod
    def INPUT_TYPES(cls):
        return {"required": {
            "batch_heads": ("INT", {"default": 1, "min": 1, "max": 40}),
            "tokens": ("INT", {"default": 9216, "min": 128, "max": 9216, "step": 64}),
            "exact_budget": ("FLOAT", {"default": 0.15625, "min": 0.015625, "max": 1.0, "step": 0.015625}),
            "dtype": (["bfloat16"], {"default": "bfloat16"}),
            "backend": (["b200", "auto", "reference"], {"default": "b200"}),
        }}

    RETURN_TYPES = ("STRING",)
    RETURN_NAMES = ("benchmark",)
    FUNCTION = "run"
    CATEGORY = "RDNA35/Attention Research"
    OUTPUT_NODE = True
    EXPERIMENTAL = True

    def run(self, batch_heads, tokens, exact_budget, dtype, backend):
        device = torch.device("cuda")
        q = torch.randn(batch_heads, tokens, 128, device=device, dtype=torch.bfloat16)
        k, v = torch.randn_like(q), torch.randn_like(q)
        ref = torch.nn.functional.scaled_dot_product_attention(q[None], k[None], v[None])[0]
        t0 = time.perf_counter()
        out, info = pisa_attention(q, k, v, exact_budget=exact_budget, backend=backend,
                                   strict_backend=backend == "b200", return_diagnostics=True)
        _sync(device)
        cold = (time.perf_counter() - t0) * 1e3
        ms = _median_ms(lambda: pisa_attention(q, k, v, exact_budget=exact_budget, backend=backend), device)
        sdpa_ms = _median_ms(lambda: torch.nn.functional.scaled_dot_product_attention(q[None], k[None], v[None]), device)
        cos = torch.nn.functional.cosine_similarity(ref.float().flatten(), out.float().flatten(), dim=0).item()
        return ("\n".join([
            "RDNA35 PISA Attention Benchmark (B200)", f"shape: BH={batch_heads} T={tokens} D=128 dtype=bfloat16",
            f"backend: {info.get('backend')}",
            f"exact blocks: {info.get('exact_blocks_per_query')}/{info.get('total_blocks')}",
            f"PISA cold call: {cold:.3f} ms", f"PISA steady-state median: {ms:.3f} ms",
            f"dense SDPA steady-state median: {sdpa_ms:.3f} ms", f"PISA/dense latency ratio: {ms / sdpa_ms:.3f}x",
            f"cosine vs dense SDPA: {cos:.9f}", f"fallback: {info.get('fallback_reason')}"]),)


class RDNA35PISARuntimeReport:
    @classmethod
    def INPUT_TYPES(cls):
        return {"required": {"model": ("MODEL",), "latent": ("LATENT",)}}

    RETURN_TYPES = ("LATENT", "STRING")
    RETURN_NAMES = ("latent", "report")
    FUNCTION = "run"
    CATEGORY = "RDNA35/Attention Research"
    OUTPUT_NODE = True
    EXPERIMENTAL = True

    def run(self, model, latent):
        state = model.get_attachment(PISA_RUNTIME_ATTACHMENT)
        if state is None:
            raise RuntimeError("RDNA35 PISA runtime state is not attached to this MODEL")
        hits = sum(state.per_layer_hits.values())
        if hits == 0:
            raise RuntimeError(f"INVALID BENCHMARK: PISA backend was not executed: {state.report()}")
        if set(state.per_layer_hits) == {-1}:
            if state.failed:
                raise RuntimeError(f"Generic PISA runtime failed: {state.report()}")
            return {"ui": {"text": [state.report()]}, "result": (latent, state.report())}
        counts = set(state.per_layer_hits.values())
        expected = set(state.expected_layers or range(ANIMA_PISA_FIRST_LAYER, ANIMA_PISA_LAST_LAYER + 1))
        if set(state.per_layer_hits) != expected or len(counts) != 1:
            raise RuntimeError(f"Incomplete PISA layer accounting: {state.report()}")
        state.verify(counts.pop())
        if not state.verified:
            raise RuntimeError(f"PISA runtime verification failed: {state.report()}")
        report = state.report()
        return {"ui": {"text": [report]}, "result": (latent, report)}


NODE_CLASS_MAPPINGS: dict[str, Any] = {
    "RDNA35BlockAttentionDiagnostics": RDNA35BlockAttentionDiagnostics,
    "RDNA35PatchModelAttention": RDNA35PatchModelAttention,
    "RDNA35PatchAnimaPISAAttention": RDNA35PatchAnimaPISAAttention,
    "RDNA35PatchMiniMaxH3GFX1151Attention": RDNA35PatchMiniMaxH3GFX1151Attention,
    "RDNA35FixedBlockAttentionBenchmark": RDNA35FixedBlockAttentionBenchmark,
    "RDNA35FullAttentionBenchmark": RDNA35FullAttentionBenchmark,
    "RDNA35MiniMaxH3GFX1151AttentionBenchmark": RDNA35MiniMaxH3GFX1151AttentionBenchmark,
    "RDNA35PISAAttentionBenchmark": RDNA35PISAAttentionBenchmark,
    "RDNA35PISARuntimeReport": RDNA35PISARuntimeReport,
}

NODE_DISPLAY_NAME_MAPPINGS = {
    "RDNA35BlockAttentionDiagnostics": "RDNA35 Block Attention Diagnostics (B200)",
    "RDNA35PatchModelAttention": "RDNA35 Patch Model Attention (B200)",
    "RDNA35PatchAnimaPISAAttention": "RDNA35 Patch PISA Attention (B200)",
    "RDNA35PatchMiniMaxH3GFX1151Attention": "RDNA35 Patch MiniMax-H3 Attention (B200)",
    "RDNA35FixedBlockAttentionBenchmark": "RDNA35 Fixed Block Attention Benchmark (B200)",
    "RDNA35FullAttentionBenchmark": "RDNA35 Exact Full Attention Benchmark (B200)",
    "RDNA35MiniMaxH3GFX1151AttentionBenchmark": "RDNA35 MiniMax-H3 Attention Benchmark (B200)",
    "RDNA35PISAAttentionBenchmark": "RDNA35 PISA Attention Benchmark (B200)",
    "RDNA35PISARuntimeReport": "RDNA35 PISA Runtime Report",
}
