"""Golden fixtures for the coverage-only step (coverage_interval < check_interval),
from the REFERENCE.

Run once, in a container that has the reference checkout (not on the GPU box):

    python tests/golden/make_golden_cv.py /path/to/coverage-verified-sparse-attention

Like make_golden.py it imports the reference's CVSABackend and runs it on CPU
tensors under TRITON_INTERPRET=1, on inputs regenerated bit-identically by
`cvsa.synthetic`. Case `small_cv_*`: the bf16 ragged case over 9 lazy steps
with check_interval=4 and coverage_interval=2, so steps 2 and 6 are
coverage-only steps of backend.py:467-520 (the gate on the page scores cached
at the last scoring step); per-step outputs, the per-step accept decisions and
the final statistics.
"""

from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))


def main(ref_root: str):
    os.environ["TRITON_INTERPRET"] = "1"
    sys.path.insert(0, ref_root)
    import torch
    torch.set_num_threads(os.cpu_count() or 8)
    from cvsa.backend import CVSABackend          # the reference's
    import importlib.util
    spec = importlib.util.spec_from_file_location(
        "b200_synthetic", os.path.join(REPO, "coverage-verified-sparse-attention_b200", "cvsa",
                                       "synthetic.py"))
    synth = importlib.util.module_from_spec(spec)
    sys.modules["b200_synthetic"] = synth      # dataclasses look their module up
    spec.loader.exec_module(synth)

    out = {}
    wl = synth.small(seed=3, B=2, Hq=8, Hkv=2, D=128, ctx=(1000, 2048))
    be = CVSABackend(num_kv_heads=2, num_q_heads=8, head_dim=128, block_size=16, num_layers=1,
                     budget_pct=wl.budget_pct, coverage_threshold=0.16, lazy=True,
                     check_interval=4, coverage_interval=2)
    g = torch.Generator().manual_seed(23)
    base = torch.randn(wl.q.shape, generator=g)
    for step in range(9):
        q = (base + 0.5 * torch.randn(wl.q.shape, generator=g)).to(wl.q.dtype)
        o = be(q, wl.k_cache, wl.v_cache, wl.block_tables, wl.context_lens, 0)
        be.step_done(0, 1)
        out[f"small_cv_q{step}"] = q.float().numpy()
        out[f"small_cv_out{step}"] = o.float().numpy()
    st = be.get_stats()
    for key in ("total_scoring_steps", "total_coverage_checks", "all_accepted_pct",
                "some_rejected_pct", "per_head_accept_rate", "effective_budget_pct"):
        out["small_cv_stat_" + key] = np.array(st[key], dtype=np.float64)

    path = os.path.join(HERE, "reference_outputs_cv.npz")
    np.savez_compressed(path, **out)
    print("wrote", path, os.path.getsize(path), "bytes")
    print({k: float(v) for k, v in out.items() if v.ndim == 0})


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit(f"usage: python {sys.argv[0]} <path to the reference checkout>")
    main(sys.argv[1])
