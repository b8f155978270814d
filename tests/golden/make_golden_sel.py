"""Golden fixtures for the reference's alternative page selectors, from the
REFERENCE.

Run once, in a container that has the reference checkout (not on the GPU box):

    python tests/golden/make_golden_sel.py /path/to/coverage-verified-sparse-attention

Like make_golden.py it imports the reference's CVSABackend and runs it on CPU
tensors under TRITON_INTERPRET=1, on inputs regenerated bit-identically by
`cvsa.synthetic` (the bf16 ragged case: B=2, Hq=8, Hkv=2, D=128, contexts
1000 and 2048 tokens, shuffled page table). Cases:

  quest_scores     CVSABackend._quest_page_scores (the Quest per-page key
                   min/max upper bound, backend.py:572-620) on the case's q.
  sel_<name>_*     a 5-step lazy run (check_interval=2) of CVSABackend with one
                   selector option: selector='quest' (selq), selector='quest'
                   with light_normalizer (ln), top_p (tp), static_budget_table
                   (staticpol), adaptive_selection (adasel), top_p with
                   approx_recovery_pct (tp_ar), and the fixed-interval
                   schedule with top_p (tp_fixed). Per step: the output,
                   the cached selection (each head's first n pages sorted) and
                   n per head, the accept mask of the last gated step; then the
                   statistics. Queries drift between steps so gates flip; the
                   tests draw them again with the same generator (seed 31:
                   base + 0.7 * N(0, 1) per step, rounded to bf16).
  rr<p>_*          random_reject_prob = 0 and 1 (the counterfactual of
                   backend.py:437-438, :490-491, :764-766): every gate forced
                   to accept / reject.
  <name>_mix       selq, ln, staticpol and adasel again at coverage_threshold
                   0.3, where some heads accept and others recover.
"""

from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))

STAT_KEYS = ("total_scoring_steps", "total_coverage_checks", "all_accepted_pct",
             "some_rejected_pct", "per_head_accept_rate", "effective_budget_pct")

# (name, extra CVSABackend keyword arguments, lazy)
CASES = [
    ("selq", dict(selector="quest"), True),
    ("ln", dict(selector="quest", light_normalizer=True), True),
    ("tp", dict(top_p=0.9), True),
    ("staticpol", dict(static_budget_table={0: [0.05, 0.25]}), True),
    ("adasel", dict(adaptive_selection=True), True),
    ("tp_ar", dict(top_p=0.6, approx_recovery_pct=0.2), True),
    ("tp_fixed", dict(top_p=0.9), False),
    ("rr0", dict(random_reject_prob=0.0), True),
    ("rr1", dict(random_reject_prob=1.0), True),
    # a lower threshold, where some heads accept and others recover
    ("selq_mix", dict(selector="quest", coverage_threshold=0.3), True),
    ("ln_mix", dict(selector="quest", light_normalizer=True, coverage_threshold=0.3), True),
    ("staticpol_mix", dict(static_budget_table={0: [0.05, 0.25]}, coverage_threshold=0.3), True),
    ("adasel_mix", dict(adaptive_selection=True, coverage_threshold=0.3), True),
]
STEPS = 5
TAU = 0.8


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
    sys.modules["b200_synthetic"] = synth
    spec.loader.exec_module(synth)

    out = {}
    wl = synth.small(seed=3, B=2, Hq=8, Hkv=2, D=128, ctx=(1000, 2048))
    be0 = CVSABackend(num_kv_heads=2, num_q_heads=8, head_dim=128, block_size=16,
                      num_layers=1, selector="quest")
    out["quest_scores"] = be0._quest_page_scores(wl.q, wl.k_cache, wl.block_tables,
                                                 wl.context_lens).numpy()

    only = os.environ.get("GOLDEN_ONLY")
    for name, kw, lazy in CASES:
        if only and name not in only.split(","):
            continue
        sched = dict(lazy=True, check_interval=2) if lazy else dict(reuse_interval=2)
        kw = dict(kw)
        tau = kw.pop("coverage_threshold", TAU)
        be = CVSABackend(num_kv_heads=2, num_q_heads=8, head_dim=128, block_size=16,
                         num_layers=1, budget_pct=wl.budget_pct, coverage_threshold=tau,
                         **sched, **kw)
        g = torch.Generator().manual_seed(31)
        base = torch.randn(wl.q.shape, generator=g)
        for step in range(STEPS):
            q = (base + 0.7 * torch.randn(wl.q.shape, generator=g)).to(wl.q.dtype)
            o = be(q, wl.k_cache, wl.v_cache, wl.block_tables, wl.context_lens, 0)
            be.step_done(0, 1)
            pi, nph = be._cached_selection[0]
            sel = np.full(tuple(pi.shape), -1, dtype=np.int32)
            for b in range(pi.shape[0]):
                for h in range(pi.shape[1]):
                    n = int(nph[b, h])
                    sel[b, h, :n] = np.sort(pi[b, h, :n].numpy())
            acc = be._last_accept_mask.get(0)
            out[f"sel_{name}_out{step}"] = o.float().numpy()
            out[f"sel_{name}_idx{step}"] = sel
            out[f"sel_{name}_n{step}"] = nph.numpy().astype(np.int32)
            out[f"sel_{name}_acc{step}"] = (np.full((2, 2), 255, dtype=np.uint8) if acc is None
                                           else acc.numpy().astype(np.uint8))
        st = be.get_stats()
        for key in STAT_KEYS:
            out[f"sel_{name}_stat_{key}"] = np.array(st[key], dtype=np.float64)
        print("case", name, "done", flush=True)

    path = os.path.join(HERE, "reference_outputs_sel.npz")
    if only and os.path.exists(path):
        # add to (or replace in) the existing fixture
        prev = dict(np.load(path))
        prev.update(out)
        out = prev
    np.savez_compressed(path, **out)
    print("wrote", path, os.path.getsize(path), "bytes")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit(f"usage: python {sys.argv[0]} <path to the reference checkout>")
    main(sys.argv[1])
