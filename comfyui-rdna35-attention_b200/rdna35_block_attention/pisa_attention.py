"""``pisa_attention`` router (mirrors the reference's
rdna35_block_attention/pisa_attention.py:38-373 API: exactly one of
exact_budget / sparsity / exact_blocks, sink_block in {0, -1, None},
backend selection, diagnostics dict).

backend="auto"/"b200" (alias "ck") runs the B200 HYD kernels on CUDA inputs
and raises if the native library is missing; "reference" is the explicit
PyTorch paper formulation (arXiv:2602.01077 eqs. 3-10: centroid routing
without the HYD bias, block-centred zeroth-order tail plus global
first-order term), which is also what CPU inputs get."""
from __future__ import annotations

import math
from typing import Any

import torch

from . import device

BLOCK_SIZE = 64
HEAD_DIM = 128
SUPPORTED_DTYPES = {torch.float16, torch.bfloat16}


def _validate_qkv(q, k, v, block_size: int) -> None:
    if not all(isinstance(x, torch.Tensor) for x in (q, k, v)):
        raise TypeError("q, k, and v must be torch tensors.")
    if q.ndim != 3:
        raise ValueError(f"PISA expects contiguous [BH,T,D] tensors, got rank {q.ndim}.")
    if q.shape != k.shape or q.shape != v.shape:
        raise ValueError(f"PISA self-attention requires identical q/k/v shapes, got {q.shape}, {k.shape}, {v.shape}.")
    if q.shape[-1] != HEAD_DIM:
        raise ValueError(f"PISA currently requires D={HEAD_DIM}, got D={q.shape[-1]}.")
    if q.shape[1] == 0:
        raise ValueError("PISA requires at least one token.")
    if q.dtype not in SUPPORTED_DTYPES or k.dtype != q.dtype or v.dtype != q.dtype:
        raise ValueError(f"PISA requires matching fp16/bf16 q/k/v, got {q.dtype}, {k.dtype}, {v.dtype}.")
    if q.device != k.device or q.device != v.device:
        raise ValueError(f"PISA requires q/k/v on one device, got {q.device}, {k.device}, {v.device}.")
    if not q.is_contiguous() or not k.is_contiguous() or not v.is_contiguous():
        raise ValueError("PISA expects contiguous q/k/v tensors.")
    if any(x.requires_grad for x in (q, k, v)):
        raise ValueError("PISA is a training-free forward prototype and does not accept tensors requiring gradients.")
    if block_size != BLOCK_SIZE:
        raise ValueError(f"PISA currently supports block_size={BLOCK_SIZE} only, got {block_size}.")


def _resolve_exact_blocks(total_blocks: int, *, exact_budget, sparsity, exact_blocks, sink_block) -> tuple[int, float]:
    if sum(x is not None for x in (exact_budget, sparsity, exact_blocks)) > 1:
        raise ValueError("Set only one of exact_budget, sparsity, or exact_blocks.")
    if exact_blocks is not None:
        if isinstance(exact_blocks, bool) or not isinstance(exact_blocks, int):
            raise TypeError("exact_blocks must be an integer.")
        if not 0 <= exact_blocks <= total_blocks:
            raise ValueError(f"exact_blocks must be in [0,{total_blocks}], got {exact_blocks}.")
        count = exact_blocks
    else:
        budget = 0.25 if exact_budget is None and sparsity is None else exact_budget
        if sparsity is not None:
            if not 0.0 <= float(sparsity) <= 1.0:
                raise ValueError(f"sparsity must be in [0,1], got {sparsity}.")
            budget = 1.0 - float(sparsity)
        if budget is None or not 0.0 <= float(budget) <= 1.0:
            raise ValueError(f"exact_budget must be in [0,1], got {budget}.")
        count = min(total_blocks, int(math.ceil(float(budget) * total_blocks)))
    if sink_block is not None:
        if sink_block not in (0, -1):
            raise ValueError("sink_block must be 0, -1, or None.")
        count = max(1, count)
    return count, count / total_blocks


def _paper_forward(q, k, v, exact_count: int, scale: float, sink_block) -> torch.Tensor:
    """Paper formulation in FP32: route on FP32 centroid scores, exact softmax
    over the chosen blocks, every other block contributes exp(q.kbar*scale)
    with weight len_j and value v_sum_j, plus the global first-order term
    (q.H*scale/T) times the tail mass, all in one normaliser."""
    bh, tokens, d = q.shape
    nb = math.ceil(tokens / BLOCK_SIZE)
    lens = torch.tensor([min(BLOCK_SIZE, tokens - i * BLOCK_SIZE) for i in range(nb)], device=q.device,
                        dtype=torch.float32)
    qf, kf, vf = q.float(), k.float(), v.float()
    pad = nb * BLOCK_SIZE - tokens
    def blocks(x):
        return torch.nn.functional.pad(x, (0, 0, 0, pad)).view(bh, nb, BLOCK_SIZE, d)
    k_mean = blocks(kf).sum(2) / lens[None, :, None]
    v_sum = blocks(vf).sum(2)
    q_mean = blocks(qf).sum(2) / lens[None, :, None]
    valid = (torch.arange(nb * BLOCK_SIZE, device=q.device) < tokens).view(nb, BLOCK_SIZE)
    centred = (blocks(kf) - k_mean[:, :, None]) * valid[None, :, :, None]
    h_sum = torch.einsum("bnrd,bnre->bde", centred, blocks(vf))
    if exact_count == nb:
        selected = torch.ones((bh, nb, nb), dtype=torch.bool, device=q.device)
    elif exact_count == 0:
        selected = torch.zeros((bh, nb, nb), dtype=torch.bool, device=q.device)
    else:
        scores = torch.einsum("bid,bjd->bij", q_mean, k_mean) * scale
        if sink_block is not None:
            scores[..., sink_block] = torch.inf
        selected = torch.zeros_like(scores, dtype=torch.bool)
        selected.scatter_(-1, torch.topk(scores, exact_count, dim=-1).indices, True)
    out = torch.empty_like(q)
    key_block = torch.arange(tokens, device=q.device) // BLOCK_SIZE
    for i in range(nb):
        s0, s1 = i * BLOCK_SIZE, min(tokens, (i + 1) * BLOCK_SIZE)
        qb = qf[:, s0:s1]
        exact_keys = selected[:, i][:, key_block]                             # [bh, T]
        logits = torch.matmul(qb, kf.transpose(1, 2)) * scale
        logits = logits.masked_fill(~exact_keys[:, None, :], -torch.inf)
        tail = torch.matmul(qb, k_mean.transpose(1, 2)) * scale + lens.log()[None, None]
        tail = tail.masked_fill(selected[:, i][:, None, :], -torch.inf)
        m = torch.maximum(logits.amax(-1), tail.amax(-1)).clamp_min(-3.0e38)
        pe = torch.exp(logits - m[..., None])
        pt = torch.exp(tail - m[..., None])                                   # includes the len_j weight
        tail_mass = pt.sum(-1, keepdim=True)
        numer = torch.matmul(pe, vf) + torch.matmul(pt / lens[None, None], v_sum)
        numer = numer + torch.matmul(qb, h_sum) * (scale / tokens) * tail_mass
        out[:, s0:s1] = (numer / (pe.sum(-1, keepdim=True) + tail_mass)).to(q.dtype)
    return out


def pisa_attention(q, k, v, *, exact_budget: float | None = None, sparsity: float | None = None,
                   exact_blocks: int | None = None, block_size: int = BLOCK_SIZE, scale: float | None = None,
                   sink_block: int | None = None, backend: str = "auto", strict_backend: bool = False,
                   return_diagnostics: bool = False):
    _validate_qkv(q, k, v, block_size)
    if backend not in {"auto", "b200", "ck", "reference"}:
        raise ValueError("backend must be one of: auto, b200 (alias: ck), reference.")
    if not isinstance(strict_backend, bool):
        raise TypeError("strict_backend must be bool.")
    total_blocks = math.ceil(q.shape[1] / block_size)
    exact_count, resolved = _resolve_exact_blocks(total_blocks, exact_budget=exact_budget, sparsity=sparsity,
                                                  exact_blocks=exact_blocks, sink_block=sink_block)
    scale_value = float(scale) if scale is not None else 1.0 / math.sqrt(q.shape[-1])
    if not math.isfinite(scale_value) or scale_value <= 0.0:
        raise ValueError(f"scale must be finite and positive, got {scale_value}.")
    used, reason = "reference", None
    if backend in {"auto", "b200", "ck"}:
        if q.device.type != "cuda":
            reason = f"b200_requires_cuda_device_not_{q.device.type}"
        elif device.b200_device_index()[0] is None:
            reason = "sm100_device_not_detected"
        elif q.dtype != torch.bfloat16 or q.shape[1] > 9216:
            reason = "b200_hyd_requires_bfloat16_and_t_le_9216"
        if reason is None:
            output = device.native_module().forward(q, k, v, exact_count, scale=scale_value, sink_block=sink_block)
            used = "b200"
        elif backend != "auto" and strict_backend:
            raise RuntimeError(f"PISA B200 backend unavailable: {reason}")
    if used == "reference":
        output = _paper_forward(q, k, v, exact_count, scale_value, sink_block)
    diagnostics: dict[str, Any] = {
        "backend": used, "requested_backend": backend, "optimized": used == "b200", "fallback_reason": reason,
        "shape": tuple(q.shape), "dtype": str(q.dtype), "block_size": block_size, "total_blocks": total_blocks,
        "exact_blocks_per_query": exact_count, "approximate_blocks_per_query": total_blocks - exact_count,
        "exact_budget": resolved, "sparsity": 1.0 - resolved, "scale": scale_value,
        "selection": "query_centroid_key_centroid_topk" + ("_hyd" if used == "b200" else ""),
        "tail_approximation": "block_centered_zeroth_plus_global_first_order", "exact_online_softmax": True,
        "shared_numerator_denominator_normalization": True, "materialized_token_qk": used != "b200",
        "routing_score_elements": q.shape[0] * total_blocks * total_blocks,
    }
    return (output, diagnostics) if return_diagnostics else output


def pisa_attention_reference(q, k, v, **kwargs):
    kwargs["backend"] = "reference"
    return pisa_attention(q, k, v, **kwargs)
