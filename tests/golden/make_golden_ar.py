"""Golden fixtures for approximate recovery (approx_recovery_pct), from the REFERENCE.

Run once, in a container that has the reference checkout (not on the GPU box):

    python tests/golden/make_golden_ar.py /path/to/coverage-verified-sparse-attention

Like make_golden.py it imports the reference's CVSABackend and runs it on CPU
tensors under TRITON_INTERPRET=1, on inputs regenerated bit-identically by
`cvsa.synthetic`. Cases (the reference's default tie-free data, no forced
pages):

  config1_ar20_*  one scoring step of config 1 with approx_recovery_pct=0.2
                  (head 1 fails tau, so the expanded top-51 branch of
                  backend.py:780-817 runs): output, expanded selection, accept
                  mask, statistics;
  small_ar20_*    the bf16 ragged case, a 4-step lazy run (check_interval=2)
                  with approx_recovery_pct=0.2 and tau=0.95: per-step outputs
                  and the final statistics.
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
    sys.path.insert(1, os.path.join(REPO, "coverage-verified-sparse-attention_b200"))
    import torch
    torch.set_num_threads(os.cpu_count() or 8)
    from cvsa.backend import CVSABackend          # the reference's (shadows ours here)
    import importlib.util
    spec = importlib.util.spec_from_file_location(
        "b200_synthetic", os.path.join(REPO, "coverage-verified-sparse-attention_b200", "cvsa",
                                       "synthetic.py"))
    synth = importlib.util.module_from_spec(spec)
    sys.modules["b200_synthetic"] = synth      # dataclasses look their module up
    spec.loader.exec_module(synth)

    out = {}
    wl1 = synth.config1()
    be = CVSABackend(num_kv_heads=2, num_q_heads=8, head_dim=64, block_size=16, num_layers=1,
                     budget_pct=wl1.budget_pct, coverage_threshold=wl1.tau,
                     approx_recovery_pct=0.2)
    o = be(wl1.q, wl1.k_cache, wl1.v_cache, wl1.block_tables, wl1.context_lens, 0)
    ei, en = be._last_expanded_selection[0]
    out["config1_ar20_output"] = o.float().numpy()
    out["config1_ar20_exp_sel"] = np.sort(ei.numpy(), axis=-1)
    out["config1_ar20_exp_n"] = en.numpy()
    out["config1_ar20_accept"] = be._last_accept_mask[0].numpy().astype(np.uint8)
    st = be.get_stats()
    out["config1_ar20_stat_effective_budget_pct"] = np.array(st["effective_budget_pct"])

    wl2 = synth.small(seed=3, B=2, Hq=8, Hkv=2, D=128, ctx=(1000, 2048))
    be = CVSABackend(num_kv_heads=2, num_q_heads=8, head_dim=128, block_size=16, num_layers=1,
                     budget_pct=wl2.budget_pct, coverage_threshold=0.95, lazy=True,
                     check_interval=2, approx_recovery_pct=0.2)
    g = torch.Generator().manual_seed(17)
    for step in range(4):
        q = torch.randn(wl2.q.shape, generator=g).to(wl2.q.dtype)
        o = be(q, wl2.k_cache, wl2.v_cache, wl2.block_tables, wl2.context_lens, 0)
        be.step_done(0, 1)
        out[f"small_ar20_q{step}"] = q.float().numpy()
        out[f"small_ar20_out{step}"] = o.float().numpy()
    st = be.get_stats()
    for key in ("total_scoring_steps", "total_coverage_checks", "per_head_accept_rate",
                "effective_budget_pct"):
        out["small_ar20_stat_" + key] = np.array(st[key], dtype=np.float64)

    path = os.path.join(HERE, "reference_outputs_ar.npz")
    np.savez_compressed(path, **out)
    print("wrote", path, os.path.getsize(path), "bytes")
    print({k: (v.shape if v.ndim else float(v)) for k, v in out.items()})


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit(f"usage: python {sys.argv[0]} <path to the reference checkout>")
    main(sys.argv[1])
