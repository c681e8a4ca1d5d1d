"""Time the reference engine's own Triton attention kernels on this GPU.

The reference's decode (kernels/decode_attention.py: load + merge) and mixed
(kernels/prefill_attention.py) kernels, JIT-compiled by Triton for the local GPU,
called through the reference's registered ops ``inference::gqa_decode_attention`` /
``inference::gqa_mixed_attention`` with its own tile configs (attn/core.py:114-137),
on the synthetic workloads ``bench.py`` times this package on (same generator,
seeds and sizes). Each point is the device time of one call with a cold L2 and
no launch gaps (``bench.graph_time_cold``). This is a measurement of the
reference, never part of the package: it imports the reference from the
unmodified copy in baseline/_ref (``install_reference.py``), in its own process,
because the reference and this package register the same op names.

Prints one JSON object: ``{"decode": [...], "mixed": {...}, "triton": version}``.
"""
from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path

REPO = Path(__file__).resolve().parents[1]


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference-copy", default=str(REPO / "baseline" / "_ref"))
    ap.add_argument("--points", default="bench",
                    help="'bench': the bench line's cases; 'sweep': configs 2 and 5 as well")
    args = ap.parse_args()
    ref = str(Path(args.reference_copy).resolve())
    sys.path.insert(0, ref)
    sys.path.insert(1, str(REPO))
    import torch
    import triton

    import attn.core as ref_core
    assert ref_core.__file__.startswith(ref), ref_core.__file__
    import bench
    from custom_inference_engine_b200 import workloads as W

    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    peak_gbs, _ = bench.measured_peak_gbs()
    peak_tf, _ = bench.bf16_peak_tflops()
    dec_op = torch.ops.inference.gqa_decode_attention.default
    mix_op = torch.ops.inference.gqa_mixed_attention.default

    out = {"triton": triton.__version__, "configs": {"decode": dict(ref_core.GQA_DECODE_CONFIG),
                                                    "mixed": dict(ref_core.GQA_PREFILL_CONFIG)},
           "timing": "cold L2 (256 MB read before each call), CUDA graph of 20 calls, "
                     "median of 5 replays minus the same graph without the calls",
           "decode": [], "mixed": {}}

    points = [(256, 4096, 0)]
    if args.points == "sweep":
        points = [(b, l, 0) for l in (512, 4096, 16384) for b in (1, 8, 64, 256)]
        points += [(8, 32768, s) for s in (4, 8, 16, 32, 64)]
    for B, L, S in points:
        c = W.make_decode_case([L] * B, seed=100 if (B, L) == (256, 4096) else 5, device=dev,
                               generate_on_device=True)
        if S:
            def fn():
                ref_core.decode_gqa_attention(
                    c.q, c.k, c.v, c.lens, c.slot_ids, c.block_table,
                    **dict(ref_core.GQA_DECODE_CONFIG, num_programs=S))
        else:
            def fn():
                dec_op(c.q, c.k, c.v, c.lens, c.slot_ids, c.block_table)
        for _ in range(3):
            fn()
        ms = bench.graph_time_cold(fn, dev)
        gbs = bench.decode_bytes(B, L) / (ms / 1e3) / 1e9
        out["decode"].append({"batch": B, "kv_len": L,
                              "num_programs": S or ref_core.GQA_DECODE_CONFIG["num_programs"],
                              "us_per_call": ms * 1e3, "gbs": gbs,
                              "frac_of_measured_hbm": gbs / peak_gbs})
        del c
        torch.cuda.empty_cache()

    if args.points == "sweep":
        # config 1: B = 8, kv_lens ~ U[1, 2048] from torch.Generator seed 0
        c = W.make_decode_case(W.config1_lens(), seed=0, device=dev, generate_on_device=True)

        def fn():
            dec_op(c.q, c.k, c.v, c.lens, c.slot_ids, c.block_table)
        for _ in range(3):
            fn()
        ms = bench.graph_time_cold(fn, dev)
        out["config1"] = {"us_per_call": ms * 1e3,
                          "gbs": c.algorithmic_bytes() / (ms / 1e3) / 1e9}
        del c

    g = torch.Generator().manual_seed(1)
    kv512 = torch.randint(0, 8193, (4,), generator=g).tolist()
    chunk3, kv3 = W.config3_shape(seed=0)
    cases = {
        "mixed_512_chunks": W.make_mixed_case([512] * 4, kv512, seed=1, device=dev,
                                              generate_on_device=True),
        "mixed_config3": W.make_mixed_case(chunk3, kv3, seed=0, device=dev, max_seqlen=2048,
                                           generate_on_device=True),
    }
    for name, c in cases.items():
        def fn(c=c):
            mix_op(c.q, c.k, c.v, max_seqlen=c.max_seqlen, cu_seqlens=c.cu_seqlens,
                   kv_lens=c.kv_lens, slot_ids=c.slot_ids, block_table=c.block_table)
        for _ in range(3):
            fn()
        ms = bench.graph_time_cold(fn, dev)
        tflops = c.causal_flops() / (ms / 1e3) / 1e12
        out["mixed"][name] = {"us_per_call": ms * 1e3, "tflops": tflops,
                              "tensor_frac": tflops / peak_tf}
    print(json.dumps(out), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
