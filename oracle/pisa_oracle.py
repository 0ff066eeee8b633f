"""CPU oracle for the B200 attention hot path -- TEST INFRASTRUCTURE ONLY.

A plain PyTorch (CPU, FP32/FP64) restatement of the reference's algorithms,
used by tests/, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
leg as the checker.  The product package never imports this module.

Each function cites the reference file:line it restates (paths inside the
ComfyUI-RDNA35-Attention project).  Pinning: tests/golden/make_golden.py
imports the reference's own Python (``_pisa_reference`` of
native/rdna35_pisa_ck/tests/test_forward.py:34-104, ``fixed_block_attention_ref``,
``pack_minimax_h3_qkv``, the generic tiling packers) and stores golden
vectors; tests/test_oracle_golden.py checks this module against them.  The
reference's own HYD forward (rdna35_pisa_ck._forward_impl) cannot run here
(HIP extension, gfx1151-only FlexAttention build), so the HYD forward is
pinned through ``_pisa_reference`` at the reference's 5e-2 tolerance, and its
pieces (stats, routing, merge) are pinned at tighter tolerances.
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F

BLOCK_SIZE = 64
SPATIAL_SIDE = 96
SPATIAL_TOKENS = SPATIAL_SIDE * SPATIAL_SIDE


# ----------------------------------------------------------------- layouts
def ordered_to_raster(ordered: torch.Tensor, grid_h: int = SPATIAL_SIDE, grid_w: int = SPATIAL_SIDE) -> torch.Tensor:
    """Block-major token index -> raster index (pisa_kernels.cu:55-64, and the
    per-frame 8x8 tiling of generic_pisa.py:17-52)."""
    frame = grid_h * grid_w
    f = ordered // frame
    o = ordered % frame
    tile = o // 64
    intra = o % 64
    tiles_per_row = grid_w // 8
    tr = tile // tiles_per_row
    tc = tile % tiles_per_row
    return f * frame + (tr * 8 + intra // 8) * grid_w + tc * 8 + intra % 8


def raster_permutation(tokens: int, grid_h: int = SPATIAL_SIDE, grid_w: int = SPATIAL_SIDE) -> torch.Tensor:
    return ordered_to_raster(torch.arange(tokens), grid_h, grid_w)


def pack_spatial(x_bhtd: torch.Tensor, grid_h: int = SPATIAL_SIDE, grid_w: int = SPATIAL_SIDE) -> torch.Tensor:
    """[B,H,T,D] raster -> [B*H,T,D] block-major (pisa_kernels.cu:247-272)."""
    b, h, t, d = x_bhtd.shape
    perm = raster_permutation(t, grid_h, grid_w)
    return x_bhtd[:, :, perm].reshape(b * h, t, d).contiguous()


def unpack_spatial(x_bh: torch.Tensor, batch: int, heads: int, grid_h: int = SPATIAL_SIDE,
                   grid_w: int = SPATIAL_SIDE) -> torch.Tensor:
    """[B*H,T,D] block-major -> [B,T,H*D] raster (pisa_kernels.cu:275-293)."""
    bh, t, d = x_bh.shape
    perm = raster_permutation(t, grid_h, grid_w)
    out = torch.empty((batch, heads, t, d), dtype=x_bh.dtype)
    out[:, :, perm] = x_bh.reshape(batch, heads, t, d)
    return out.permute(0, 2, 1, 3).reshape(batch, t, heads * d)


def block_lengths(tokens: int) -> list[int]:
    blocks = (tokens + BLOCK_SIZE - 1) // BLOCK_SIZE
    return [min(BLOCK_SIZE, tokens - i * BLOCK_SIZE) for i in range(blocks)]


def _seq_sum(x: torch.Tensor) -> torch.Tensor:
    """FP32 sum over dim 1 in row order (the per-dim loop of pisa_kernels.cu:191-200)."""
    acc = torch.zeros((x.shape[0], x.shape[2]), dtype=torch.float32)
    for r in range(x.shape[1]):
        acc = acc + x[:, r].float()
    return acc


# ----------------------------------------------------------------- statistics
def hyd_block_stats(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor):
    """HYD statistics of pisa_kernels.cu:167-244 on [BH,T,D]:
    (q_centroids BF16, k_centroids FP32, v_means BF16, h_sum FP32, h_norm FP32).
    Centroids: sequential FP32 sums times float(1/len) (bit-exact to the
    kernel).  H_blk = sum_r (k_r - kbar) v_r^T with FP32-centred K, evaluated
    in FP64 and rounded (the reference accumulates in FP32; both are within
    the 1e-3 relative gate of test_forward.py:181-201)."""
    bh, tokens, d = q.shape
    lens = block_lengths(tokens)
    qc, kc, vc, norms = [], [], [], []
    h_sum = torch.zeros((bh, d, d), dtype=torch.float64)
    for blk, ln in enumerate(lens):
        s = blk * BLOCK_SIZE
        inv = torch.tensor(1.0, dtype=torch.float32) / torch.tensor(float(ln), dtype=torch.float32)
        qm = _seq_sum(q[:, s:s + ln]) * inv
        km = _seq_sum(k[:, s:s + ln]) * inv
        vm = _seq_sum(v[:, s:s + ln]) * inv
        qc.append(qm.to(q.dtype))
        kc.append(km)
        vc.append(vm.to(v.dtype))
        centred = (k[:, s:s + ln].float() - km[:, None, :]).double()
        h_blk = torch.bmm(centred.transpose(1, 2), v[:, s:s + ln].double())
        h_sum += h_blk
        norms.append(torch.linalg.matrix_norm(h_blk).float())
    return (torch.stack(qc, 1), torch.stack(kc, 1), torch.stack(vc, 1), h_sum.float(), torch.stack(norms, 1))


def generic_block_stats(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor):
    """Generic statistics (generic_pisa.py:106-138 fallback + pisa_kernel.py:49-84):
    (q_centroids FP32 = sum/len, k_centroids FP32 = sum/len, v_sums FP32,
    h_sum FP32 with the centred K rounded to the input dtype, lengths)."""
    bh, tokens, d = q.shape
    lens = block_lengths(tokens)
    qc, kc, vs = [], [], []
    h_sum = torch.zeros((bh, d, d), dtype=torch.float64)
    for blk, ln in enumerate(lens):
        s = blk * BLOCK_SIZE
        qf = q[:, s:s + ln].float()
        kf = k[:, s:s + ln].float()
        vf = v[:, s:s + ln].float()
        qc.append(qf.sum(1) / ln)
        km = kf.sum(1) / ln
        kc.append(km)
        vs.append(vf.sum(1))
        centred = (kf - km[:, None]).to(k.dtype).double()
        h_sum += torch.bmm(centred.transpose(1, 2), vf.double())
    return (torch.stack(qc, 1), torch.stack(kc, 1), torch.stack(vs, 1), h_sum.float(),
            torch.tensor(lens, dtype=torch.float32))


# ----------------------------------------------------------------- routing
def route_scores_hyd(q_centroids: torch.Tensor, k_centroids: torch.Tensor, h_norm: torch.Tensor,
                     scale: float) -> torch.Tensor:
    """rdna35_pisa_ck/__init__.py:258-261: bmm(BF16 qc, BF16 kc^T) in FP32,
    *scale, + log(h_norm + 1e-5)."""
    qcb = q_centroids.to(torch.bfloat16).double()
    kcb = k_centroids.to(torch.bfloat16).double()
    s = torch.bmm(qcb, kcb.transpose(1, 2)).float()
    s = s * torch.tensor(scale, dtype=torch.float32)
    return s + torch.log(h_norm[:, None, :] + torch.tensor(1e-5, dtype=torch.float32))


def route_scores_generic(q_centroids: torch.Tensor, k_centroids: torch.Tensor, scale: float) -> torch.Tensor:
    """generic_pisa.py:172-173: FP32 bmm of FP32 centroids, *scale."""
    s = torch.bmm(q_centroids.double(), k_centroids.double().transpose(1, 2)).float()
    return s * torch.tensor(scale, dtype=torch.float32)


def select_topk(scores: torch.Tensor, exact_blocks: int, sink_block: int | None = None) -> torch.Tensor:
    """topk(k).indices.sort() (rdna35_pisa_ck/__init__.py:262-264); ties at the
    cut resolve to the lower index."""
    scores = scores.clone()
    if sink_block is not None:
        scores[..., sink_block] = torch.inf
    order = torch.sort(-scores, dim=-1, stable=True).indices
    return order[..., :exact_blocks].sort(dim=-1).values


def near_tie_rows(scores: torch.Tensor, exact_blocks: int, rel: float = 1e-5, abs_tol: float = 0.0) -> torch.Tensor:
    """Rows whose k-th and (k+1)-th largest scores lie within
    rel*max(1,|s|) + abs_tol: index sets there may legitimately differ between
    implementations.  abs_tol carries a bound on the per-column score error
    of the implementation under test (e.g. twice its max |d log h_norm|)."""
    if exact_blocks <= 0 or exact_blocks >= scores.shape[-1]:
        return torch.zeros(scores.shape[:-1], dtype=torch.bool)
    top = torch.topk(scores, exact_blocks + 1, dim=-1).values
    a, b = top[..., exact_blocks - 1], top[..., exact_blocks]
    return (a - b).abs() <= rel * torch.clamp(a.abs(), min=1.0) + abs_tol


# ----------------------------------------------------------------- attention
def _softmax_attend(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float, mask=None):
    """FP32 softmax attention returning (out, natural-log LSE)."""
    s = torch.matmul(q.float(), k.float().transpose(-1, -2)) * scale
    if mask is not None:
        s = s.masked_fill(~mask, -torch.inf)
    lse = torch.logsumexp(s, dim=-1)
    p = torch.exp(s - lse[..., None])
    return torch.matmul(p, v.float()), lse


def hyd_forward(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, exact_blocks: int, scale: float | None = None,
                sink_block: int | None = None, stats=None):
    """PISA HYD forward on [BH,T,128] (rdna35_pisa_ck/__init__.py:233-316):
    exact block-sparse attention over the routed blocks + centroid tail
    (logit q.kc*scale + log len, selected masked) + correction
    q.bf16(h_sum)*scale/T, merged with LSE weights.  The exact and tail outputs
    are rounded to the input dtype before the merge, as FlexAttention returns
    them.  Returns (output, indices)."""
    bh, tokens, d = q.shape
    nb = (tokens + BLOCK_SIZE - 1) // BLOCK_SIZE
    scale = 1.0 / math.sqrt(d) if scale is None else float(scale)
    scale = float(torch.tensor(scale, dtype=torch.float32))
    if exact_blocks == nb:
        out, _ = _softmax_attend(q, k, v, scale)
        return out.to(q.dtype), torch.arange(nb).expand(bh, nb, nb)
    qc, kc, vc, h_sum, h_norm = stats if stats is not None else hyd_block_stats(q, k, v)
    if exact_blocks > 0:
        indices = select_topk(route_scores_hyd(qc, kc, h_norm, scale), exact_blocks, sink_block)
    else:
        indices = torch.empty((bh, nb, 0), dtype=torch.int64)
    lens = torch.tensor(block_lengths(tokens), dtype=torch.float32)
    kcb = kc.to(q.dtype).float()
    out = torch.empty((bh, tokens, d), dtype=torch.float32)
    corr_all = torch.matmul(q.float(), h_sum.to(q.dtype).float()) * torch.tensor(scale / tokens, dtype=torch.float32)
    for b in range(bh):
        for i in range(nb):
            s0, s1 = i * BLOCK_SIZE, min(tokens, (i + 1) * BLOCK_SIZE)
            qb = q[b, s0:s1].float()
            sel = indices[b, i].tolist()
            # tail
            tail = (qb @ kcb[b].T) * scale + lens.log()[None]
            selected = torch.zeros(nb, dtype=torch.bool)
            selected[sel] = True
            tail = tail.masked_fill(selected[None], -torch.inf)
            tail_lse = torch.logsumexp(tail, -1)
            tail_out = (torch.exp(tail - tail_lse[:, None]) @ vc[b].float()).to(q.dtype).float()
            corr = corr_all[b, s0:s1]
            if exact_blocks == 0:
                out[b, s0:s1] = tail_out + corr
                continue
            rows = torch.cat([torch.arange(j * BLOCK_SIZE, min(tokens, (j + 1) * BLOCK_SIZE)) for j in sel])
            ex_out, ex_lse = _softmax_attend(qb, k[b, rows], v[b, rows], scale)
            ex_out = ex_out.to(q.dtype).float()
            total = torch.logaddexp(ex_lse, tail_lse)
            we = torch.exp(ex_lse - total)[:, None]
            wa = torch.exp(tail_lse - total)[:, None]
            out[b, s0:s1] = ex_out * we + tail_out * wa + corr * wa
    return out.to(q.dtype), indices


def _blocked_sparse_forward(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, indices: torch.Tensor,
                            tail_keys: torch.Tensor, tail_values: torch.Tensor, tail_bias: torch.Tensor,
                            correction: torch.Tensor | None, scale: float, chunk: int = 32) -> torch.Tensor:
    """Batched form of the per-query-block loops of hyd_forward /
    generic_forward for one (batch, head): the selected key rows of every
    query block are gathered at once (chunks of ``chunk`` query blocks) and
    the exact, tail and correction terms are merged with LSE weights exactly
    as those loops do (exact and tail outputs rounded to q.dtype first).
    q/k/v: [T,D]; indices [nb,kx]; tail_keys [nb,D] (already rounded);
    tail_values [nb,D] FP32; tail_bias [nb] added to every tail logit;
    correction [T,D] FP32 or None.  Returns FP32 [T,D]."""
    tokens, d = q.shape
    nb = indices.shape[0]
    kx = indices.shape[1]
    pad = nb * BLOCK_SIZE - tokens
    qf = F.pad(q.float(), (0, 0, 0, pad)).view(nb, BLOCK_SIZE, d)
    kf = F.pad(k.float(), (0, 0, 0, pad))
    vf = F.pad(v.float(), (0, 0, 0, pad))
    out = torch.empty((nb, BLOCK_SIZE, d), dtype=torch.float32)
    sel_mask = torch.zeros((nb, nb), dtype=torch.bool)
    if kx:
        sel_mask.scatter_(1, indices.long(), True)
    lane = torch.arange(BLOCK_SIZE)
    corr = None if correction is None else F.pad(correction, (0, 0, 0, pad)).view(nb, BLOCK_SIZE, d)
    for c0 in range(0, nb, chunk):
        c1 = min(nb, c0 + chunk)
        qb = qf[c0:c1]
        tail = torch.matmul(qb, tail_keys.T) * scale + tail_bias[None, None]
        tail = tail.masked_fill(sel_mask[c0:c1, None, :], -torch.inf)
        tail_lse = torch.logsumexp(tail, -1)
        tail_out = torch.matmul(torch.exp(tail - tail_lse[..., None]), tail_values).to(q.dtype).float()
        wa_corr = corr[c0:c1] if corr is not None else None
        if kx == 0:
            o = tail_out if wa_corr is None else tail_out + wa_corr
        else:
            rows = (indices[c0:c1].long()[..., None] * BLOCK_SIZE + lane).reshape(c1 - c0, kx * BLOCK_SIZE)
            s = torch.bmm(qb, kf[rows].transpose(1, 2)) * scale
            s = s.masked_fill((rows >= tokens)[:, None, :], -torch.inf)
            ex_lse = torch.logsumexp(s, -1)
            ex_out = torch.bmm(torch.exp(s - ex_lse[..., None]), vf[rows]).to(q.dtype).float()
            total = torch.logaddexp(ex_lse, tail_lse)
            we = torch.exp(ex_lse - total)[..., None]
            wa = torch.exp(tail_lse - total)[..., None]
            o = ex_out * we + tail_out * wa
            if wa_corr is not None:
                o = o + wa_corr * wa
        out[c0:c1] = o
    return out.view(nb * BLOCK_SIZE, d)[:tokens]


def hyd_forward_batched(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, exact_blocks: int,
                        scale: float | None = None, sink_block: int | None = None, stats=None, heads=None):
    """hyd_forward with the per-query-block loop replaced by gathered batched
    matmuls (the shape of the reference's own torch ops,
    rdna35_pisa_ck/__init__.py:254-316).  Same semantics and return value;
    ``heads`` restricts the attention to those rows of the [BH,...] inputs
    (their outputs only; other rows of the result are left zero)."""
    bh, tokens, d = q.shape
    nb = (tokens + BLOCK_SIZE - 1) // BLOCK_SIZE
    scale = 1.0 / math.sqrt(d) if scale is None else float(scale)
    scale = float(torch.tensor(scale, dtype=torch.float32))
    if exact_blocks == nb:
        out, _ = _softmax_attend(q, k, v, scale)
        return out.to(q.dtype), torch.arange(nb).expand(bh, nb, nb)
    qc, kc, vc, h_sum, h_norm = stats if stats is not None else hyd_block_stats(q, k, v)
    if exact_blocks > 0:
        indices = select_topk(route_scores_hyd(qc, kc, h_norm, scale), exact_blocks, sink_block)
    else:
        indices = torch.empty((bh, nb, 0), dtype=torch.int64)
    log_lens = torch.tensor(block_lengths(tokens), dtype=torch.float32).log()
    kcb = kc.to(q.dtype).float()
    out = torch.zeros((bh, tokens, d), dtype=torch.float32)
    corr_scale = torch.tensor(scale / tokens, dtype=torch.float32)
    for b in (range(bh) if heads is None else heads):
        corr = torch.matmul(q[b].float(), h_sum[b].to(q.dtype).float()) * corr_scale
        out[b] = _blocked_sparse_forward(q[b], k[b], v[b], indices[b], kcb[b], vc[b].float(), log_lens, corr, scale)
    return out.to(q.dtype), indices


def hyd_forward_spatial(q_bhtd: torch.Tensor, k_bhtd: torch.Tensor, v_bhtd: torch.Tensor, exact_blocks: int,
                        scale: float | None = None, sink_block: int | None = None):
    """forward_spatial_bhtd (rdna35_pisa_ck/__init__.py:344-365): pack, HYD
    forward, raster output [B,T,H*D]."""
    b, h, t, d = q_bhtd.shape
    packed = [pack_spatial(x) for x in (q_bhtd, k_bhtd, v_bhtd)]
    out, idx = hyd_forward(*packed, exact_blocks, scale, sink_block)
    return unpack_spatial(out, b, h), idx


def generic_forward(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, exact_blocks: int, scale: float | None = None,
                    use_first_order: bool = True):
    """generic_pisa_attention (generic_pisa.py:141-232) on [BH,T,D], with the
    Triton-statistics semantics (generic_pisa.py:120-138).  Returns (out, idx)."""
    bh, tokens, d = q.shape
    nb = (tokens + BLOCK_SIZE - 1) // BLOCK_SIZE
    scale = 1.0 / math.sqrt(d) if scale is None else float(scale)
    if exact_blocks == nb:
        out, _ = _softmax_attend(q, k, v, scale)
        return out.to(q.dtype), torch.arange(nb).expand(bh, nb, nb)
    qc, kc, vsum, h_sum, lens = generic_block_stats(q, k, v)
    vmean = vsum / lens[None, :, None]
    indices = select_topk(route_scores_generic(qc, kc, scale), exact_blocks)
    kcb = kc.to(q.dtype).float()
    out = torch.empty((bh, tokens, d), dtype=torch.float32)
    corr_all = None
    if use_first_order:
        corr_all = torch.matmul(q.float(), h_sum.to(q.dtype).float()) * (scale / tokens)
    for b in range(bh):
        for i in range(nb):
            s0, s1 = i * BLOCK_SIZE, min(tokens, (i + 1) * BLOCK_SIZE)
            qb = q[b, s0:s1].float()
            sel = indices[b, i].tolist()
            tail = (qb @ kcb[b].T) * scale
            selected = torch.zeros(nb, dtype=torch.bool)
            selected[sel] = True
            tail = tail.masked_fill(selected[None], -torch.inf) + lens.log()[None]
            tail_lse = torch.logsumexp(tail, -1)
            tail_out = (torch.softmax(tail, -1) @ vmean[b]).to(q.dtype).float()
            rows = torch.cat([torch.arange(j * BLOCK_SIZE, min(tokens, (j + 1) * BLOCK_SIZE)) for j in sel])
            ex_out, ex_lse = _softmax_attend(qb, k[b, rows], v[b, rows], scale)
            ex_out = ex_out.to(q.dtype).float()
            total = torch.logaddexp(ex_lse, tail_lse)
            we = torch.exp(ex_lse - total)[:, None]
            wa = torch.exp(tail_lse - total)[:, None]
            o = ex_out * we + tail_out * wa
            if corr_all is not None:
                o = o + corr_all[b, s0:s1] * wa
            out[b, s0:s1] = o
    return out.to(q.dtype), indices


def generic_forward_batched(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, exact_blocks: int,
                            scale: float | None = None, use_first_order: bool = True, heads=None):
    """generic_forward with gathered batched matmuls in place of its
    per-query-block loop; same semantics.  ``heads`` as in hyd_forward_batched."""
    bh, tokens, d = q.shape
    nb = (tokens + BLOCK_SIZE - 1) // BLOCK_SIZE
    scale = 1.0 / math.sqrt(d) if scale is None else float(scale)
    if exact_blocks == nb:
        out, _ = _softmax_attend(q, k, v, scale)
        return out.to(q.dtype), torch.arange(nb).expand(bh, nb, nb)
    qc, kc, vsum, h_sum, lens = generic_block_stats(q, k, v)
    vmean = vsum / lens[None, :, None]
    indices = select_topk(route_scores_generic(qc, kc, scale), exact_blocks)
    kcb = kc.to(q.dtype).float()
    out = torch.zeros((bh, tokens, d), dtype=torch.float32)
    for b in (range(bh) if heads is None else heads):
        corr = None
        if use_first_order:
            corr = torch.matmul(q[b].float(), h_sum[b].to(q.dtype).float()) * (scale / tokens)
        out[b] = _blocked_sparse_forward(q[b], k[b], v[b], indices[b], kcb[b], vmean[b], lens.log(), corr, scale)
    return out.to(q.dtype), indices


def merge_epilogue(exact, exact_lse, approx, approx_lse, correction):
    """pisa_kernels.cu:317-339 (block-major; unpack separately)."""
    mx = torch.maximum(exact_lse, approx_lse)
    total = mx + torch.log(torch.exp(exact_lse - mx) + torch.exp(approx_lse - mx))
    we = torch.exp(exact_lse - total)[..., None]
    wa = torch.exp(approx_lse - total)[..., None]
    return (exact.float() * we + approx.float() * wa + correction * wa).to(exact.dtype)


def full_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float | None = None):
    """Exact attention (triton_kernel.py:113-160; F.scaled_dot_product_attention
    math) in FP32 over [..., T, D]; returns (out in q.dtype, LSE)."""
    scale = 1.0 / math.sqrt(q.shape[-1]) if scale is None else float(scale)
    out, lse = _softmax_attend(q, k, v, scale)
    return out.to(q.dtype), lse


def fixed_block_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float | None = None,
                          causal: bool = False, block_size: int = BLOCK_SIZE, round_p: bool = False,
                          mask: torch.Tensor | None = None):
    """reference.py:159-200 on [..., T, D]: each 64-token query block attends to
    its own key block, FP32.  round_p=True rounds P to the input dtype before
    P.V, as the 16-bit Triton kernel does (triton_kernel.py:96).  mask: a
    tensor broadcastable to [..., T, T] (reference.py:114-156 after its
    rank rules): boolean masks keep True entries, others are added to the
    scaled scores after the causal mask; a fully masked row gives NaN."""
    t, d = q.shape[-2], q.shape[-1]
    scale = 1.0 / math.sqrt(d) if scale is None else float(scale)
    out = torch.empty(q.shape, dtype=torch.float32)
    for s in range(0, t, block_size):
        e = min(s + block_size, t)
        sc = torch.matmul(q[..., s:e, :].float(), k[..., s:e, :].float().transpose(-1, -2)) * scale
        if causal:
            m = torch.ones((e - s, e - s), dtype=torch.bool).triu(1)
            sc = sc.masked_fill(m, -torch.inf)
        if mask is not None:
            blk = mask[..., s:e, s:e]
            sc = sc.masked_fill(~blk, -torch.inf) if blk.dtype == torch.bool else sc + blk.float()
        p = torch.softmax(sc, dim=-1)
        if round_p:
            p = p.to(q.dtype).float()
        out[..., s:e, :] = torch.matmul(p, v[..., s:e, :].float())
    return out.to(q.dtype)


def h3_pack(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, pack_all_tokens: int = 12000):
    """pack_minimax_h3_qkv (minimax_h3_gfx1151_attention.py:64-74)."""
    if q.shape[2] >= pack_all_tokens:
        packed = torch.stack((q, k, v))
        return packed[0], packed[1], packed[2], "qkv"
    packed = torch.stack((k, v))
    return q, packed[0], packed[1], "kv"


# ----------------------------------------------------------------- inputs
def anima_inputs(batch: int = 2, heads: int = 16, seed: int = 0, side: int = SPATIAL_SIDE, dtype=torch.bfloat16,
                 offset_sigma: float = 0.5):
    """Config-3 synthetic inputs: Q,K,V raster [B,T,H,128] = N(0,1) plus a
    per-(b,h,8x8 tile,d) offset N(0, offset_sigma) constant over the tile.
    Returns BHTD views of the BTHD storage (the Anima attn_op contract)."""
    tokens = side * side
    tiles = (side // 8) ** 2
    perm = raster_permutation(tokens, side, side)
    gen = torch.Generator().manual_seed(seed)
    outs = []
    for _ in range(3):
        base = torch.randn((batch, heads, tokens, 128), generator=gen)
        off = torch.randn((batch, heads, tiles, 1, 128), generator=gen) * offset_sigma
        ordered = base.view(batch, heads, tiles, 64, 128) + off
        raster = torch.empty_like(base)
        raster[:, :, perm] = ordered.view(batch, heads, tokens, 128)
        bthd = raster.permute(0, 2, 1, 3).contiguous().to(dtype)
        outs.append(bthd.permute(0, 2, 1, 3))
    return tuple(outs)


def generic_inputs(bh: int, tokens: int, seed: int = 0, dtype=torch.bfloat16, offset_sigma: float = 0.5):
    """Config-5 synthetic inputs: [BH,T,128] N(0,1) + per-(bh,64-token block,d)
    offsets N(0, offset_sigma) in block-major order."""
    nb = (tokens + BLOCK_SIZE - 1) // BLOCK_SIZE
    gen = torch.Generator().manual_seed(seed)
    outs = []
    for _ in range(3):
        base = torch.randn((bh, nb * BLOCK_SIZE, 128), generator=gen)
        off = torch.randn((bh, nb, 1, 128), generator=gen) * offset_sigma
        x = (base.view(bh, nb, BLOCK_SIZE, 128) + off).view(bh, nb * BLOCK_SIZE, 128)[:, :tokens]
        outs.append(x.contiguous().to(dtype))
    return tuple(outs)
