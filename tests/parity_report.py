"""Measured parity of the attention outputs per benchmark configuration (BASELINE.json configs[0..3]), both paths:
per-row cosine and max-abs error of the GPU output against float64 softmax of the same inputs and against the
oracle's restatement of the same arithmetic, on 4,096 rows spread over every head and over positions (first and last
rows included). Prints one markdown table. Needs a GPU; run from the repo root: ``python tests/parity_report.py``.

Test infrastructure (the numbers the parity statement quotes); the pass/fail bounds are in tests/test_gpu_*.py."""
from __future__ import annotations

import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
for p in (ROOT, os.path.join(ROOT, "oracle"), HERE):
    if p not in sys.path:
        sys.path.insert(0, p)

CONFIGS = [("c0", 2048, 8), ("c1", 2159, 32), ("c2", 16848, 32), ("c3", 47232, 32)]


def main() -> None:
    import torch

    from _util import attention_stats, run_attention, sample_rows
    from sycl_minimax_h3_b200.workloads import make_qkv

    dev = torch.device("cuda", 0)
    D = 128
    print("| config | S x H | path | rows | min cos vs float64 | max-abs vs float64 | min cos vs same semantics | "
          "max-abs vs same semantics |")
    print("|---|---|---|---|---|---|---|---|")
    for name, S, H in CONFIGS:
        qkv = make_qkv(S, H, D, seed=S + 11)
        dq = qkv.to(dev)
        rows = sample_rows(S, H, 4096, seed=S)
        for path, min_s in (("Sage int8", 0), ("fp16 SDPA", 1 << 30)):
            out = run_attention(dq, H, D, min_s=min_s)
            st = attention_stats(qkv, out, H, D, sage=min_s == 0, rows=rows)
            print(f"| {name} | {S:,} x {H} | {path} | {st['rows']} | {st['min_cos_vs_exact']:.6f} | "
                  f"{st['max_abs_vs_exact']:.3e} | {st['min_cos_vs_same_semantics']:.6f} | "
                  f"{st['max_abs_vs_same_semantics']:.3e} |", flush=True)


if __name__ == "__main__":
    main()
