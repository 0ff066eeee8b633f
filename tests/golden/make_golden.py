"""Generate the golden vectors that pin the CPU oracle to the reference.

Run in the container that has the reference checkout (read-only):
    python tests/golden/make_golden.py /path/to/ComfyUI-RDNA35-Attention
It imports the reference's own Python implementations -- never the product
package -- and writes tests/golden/golden.pt:
  * fixed_block: rdna35_block_attention.reference.fixed_block_attention_ref
    (config 1 shape scaled to 2 heads x 256 tokens; plain and causal), and
    fixed_block_masked: the same with [T,T] / [N,T,T] / [B,H,T,T] boolean and
    additive float masks (ragged T=130, causal, fully masked rows -> NaN);
  * pisa_hyd: _pisa_reference of native/rdna35_pisa_ck/tests/test_forward.py
    (the reference's own pure-torch HYD oracle; the native wheel it imports
    is stubbed because it cannot load without its ROCm build) for T in
    {65, 128, 256} with exact_blocks 0/1/2 and sink blocks, and at the full
    Anima size T=9216 with 23 of 144 exact blocks (every 8th output row);
  * pisa_paper: pisa_attention(backend="reference") (paper variant);
  * h3_pack: pack_minimax_h3_qkv value/identity checks;
  * tiling: generic_pisa._pack_spatial_blocks / _pack_video_blocks
    permutations.
Inputs are regenerated from the seeds stored next to each case.
"""
from __future__ import annotations

import importlib.util
import pathlib
import sys
import types

import torch


def seeded(shape, seed, dtype=torch.float32):
    gen = torch.Generator().manual_seed(seed)
    return torch.randn(shape, generator=gen).to(dtype)


MASK_CASES = [
    {"name": "bool_2d", "shape": (130, 130), "kind": "bool", "causal": False, "seed": 500},
    {"name": "bool_3d_per_batch", "shape": (1, 130, 130), "kind": "bool", "causal": True, "seed": 510},
    {"name": "bool_4d_per_head", "shape": (1, 2, 130, 130), "kind": "bool", "causal": False, "seed": 520},
    {"name": "float_3d_per_bh", "shape": (2, 130, 130), "kind": "float", "causal": False, "seed": 530},
    {"name": "bool_2d_dead_rows", "shape": (130, 130), "kind": "bool_dead_rows", "causal": False, "seed": 540},
]


def make_mask(case):
    """The mask of one masked case, regenerated from its seed (bool: keep
    ~70% of entries; float: N(0,1) terms; dead rows: rows 3 and 70 masked
    entirely)."""
    gen = torch.Generator().manual_seed(case["seed"] + 99)
    if case["kind"] == "float":
        return torch.randn(case["shape"], generator=gen)
    mask = torch.rand(case["shape"], generator=gen) > 0.3
    if case["kind"] == "bool_dead_rows":
        mask[3] = False
        mask[70] = False
    return mask


def block_offset_inputs(tokens, seed, dtype=torch.bfloat16):
    """[1,T,128] N(0,1) plus a per-64-token-block N(0,0.5) offset (config 3's
    value distribution in block-major order)."""
    blocks = (tokens + 63) // 64
    base = seeded((1, blocks * 64, 128), seed)
    off = seeded((1, blocks, 1, 128), seed + 100000) * 0.5
    return (base.view(1, blocks, 64, 128) + off).view(1, blocks * 64, 128)[:, :tokens].contiguous().to(dtype)


def main(ref_root: str) -> None:
    sys.path.insert(0, ref_root)
    sys.modules["rdna35_pisa_ck"] = types.ModuleType("rdna35_pisa_ck")  # stub: ROCm-only wheel
    from rdna35_block_attention.generic_pisa import _pack_spatial_blocks, _pack_video_blocks
    from rdna35_block_attention.minimax_h3_gfx1151_attention import pack_minimax_h3_qkv
    from rdna35_block_attention.pisa_attention import pisa_attention
    from rdna35_block_attention.reference import fixed_block_attention_ref

    spec = importlib.util.spec_from_file_location(
        "ref_test_forward", pathlib.Path(ref_root) / "native/rdna35_pisa_ck/tests/test_forward.py")
    test_forward = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(test_forward)
    pisa_reference = test_forward._pisa_reference

    golden: dict = {"fixed_block": [], "fixed_block_masked": [], "pisa_hyd": [], "pisa_hyd_full": [], "pisa_paper": [], "tiling": {}, "h3_pack": {}}
    for causal in (False, True):
        q, k, v = (seeded((1, 2, 256, 64), 100 + i) for i in range(3))
        out = fixed_block_attention_ref(q, k, v, block_size=64, scale=0.125, causal=causal, layout="bhtd")
        golden["fixed_block"].append({"seeds": (100, 101, 102), "shape": (1, 2, 256, 64), "scale": 0.125,
                                      "causal": causal, "out": out})
    # masked fixed-block cases (reference.py:114-200): mask forms by rank,
    # bool and additive float, with causal, ragged T and fully masked rows
    for case in MASK_CASES:
        q, k, v = (seeded((1, 2, 130, 32), case["seed"] + i) for i in range(3))
        mask = make_mask(case)
        out = fixed_block_attention_ref(q, k, v, block_size=64, scale=None, causal=case["causal"], layout="bhtd",
                                        mask=mask)
        golden["fixed_block_masked"].append({**case, "out": out})
    for tokens, exact, sink, seed in ((128, 1, None, 19), (65, 1, 0, 23), (65, 1, -1, 23), (256, 2, None, 31),
                                      (256, 0, None, 37), (128, 2, None, 17)):
        q, k, v = (seeded((1, tokens, 128), seed * 10 + i, torch.bfloat16) for i in range(3))
        out = pisa_reference(q, k, v, exact_blocks=exact, sink_block=sink)
        golden["pisa_hyd"].append({"seeds": tuple(seed * 10 + i for i in range(3)), "tokens": tokens,
                                   "exact_blocks": exact, "sink_block": sink, "out": out.to(torch.bfloat16)})
    # full Anima block count (144 blocks, the 23-block cut) on block-offset
    # inputs so the routing is non-trivial; every 8th output row is stored
    for tokens, exact, sink, seed in ((9216, 23, None, 71), (9216, 23, 0, 73)):
        q, k, v = (block_offset_inputs(tokens, seed * 10 + i) for i in range(3))
        out = pisa_reference(q, k, v, exact_blocks=exact, sink_block=sink)
        golden["pisa_hyd_full"].append({"seeds": tuple(seed * 10 + i for i in range(3)), "tokens": tokens,
                                        "exact_blocks": exact, "sink_block": sink, "row_step": 8,
                                        "out_rows": out[:, ::8].to(torch.bfloat16).clone()})
    for tokens, exact, seed in ((256, 2, 41), (200, 1, 43)):
        q, k, v = (seeded((2, tokens, 128), seed * 10 + i, torch.bfloat16) for i in range(3))
        out = pisa_attention(q, k, v, exact_blocks=exact, backend="reference")
        golden["pisa_paper"].append({"seeds": tuple(seed * 10 + i for i in range(3)), "bh": 2, "tokens": tokens,
                                     "exact_blocks": exact, "out": out})
    x = torch.arange(256).reshape(1, 1, 256, 1)
    golden["tiling"]["spatial_16"] = _pack_spatial_blocks(x, 16).flatten()
    x = torch.arange(9216).reshape(1, 1, 9216, 1)
    golden["tiling"]["spatial_96"] = _pack_spatial_blocks(x, 96).flatten()
    x = torch.arange(2 * 32 * 64).reshape(1, 1, 2 * 32 * 64, 1)
    golden["tiling"]["video_2_32_64"] = _pack_video_blocks(x, (2, 32, 64)).flatten()
    qkv = torch.arange(1 * 12000 * 3, dtype=torch.float32).reshape(1, 12000, 3, 1, 1)
    views = [qkv[:, :, i].permute(0, 2, 1, 3) for i in range(3)]
    pq, pk, pv, profile = pack_minimax_h3_qkv(*views)
    golden["h3_pack"] = {"profile_12000": profile, "sum": float(pq.sum() + 2 * pk.sum() + 3 * pv.sum())}
    out_path = pathlib.Path(__file__).resolve().parent / "golden.pt"
    torch.save(golden, out_path)
    print(f"wrote {out_path} ({out_path.stat().st_size} bytes)")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py <path of the reference checkout>")
    main(sys.argv[1])
