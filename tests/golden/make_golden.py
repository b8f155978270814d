"""Generate the golden fixtures by running the REFERENCE implementation.

Run once, in a container that has the reference checkout (not on the GPU box):

    python tests/golden/make_golden.py /path/to/coverage-verified-sparse-attention

It imports the reference's own Triton kernels and CVSABackend and runs them on
CPU tensors under TRITON_INTERPRET=1 (Triton's interpreter), on seeded
synthetic inputs regenerated bit-identically by `cvsa.synthetic` (CPU
generators). Only outputs are stored (a few KB per case) plus a checksum of
the inputs, so the tests can regenerate and verify the inputs. Cases:

  config1_*   BASELINE config 1 (fp32, D=64, 256 pages): the reference's page
              scores; its decode / coverage / complement / merge on the
              oracle's extended selection (forced pages + stable top-32); and
              one full reference CVSABackend scoring step (no forced pages).
  small_*     bf16, D=128, ragged contexts (1000, 2048 tokens), shuffled page
              table: the same kernel outputs; plus a 5-step lazy CVSABackend
              run (check_interval=2) with the reference's per-step outputs.
"""

from __future__ import annotations

import hashlib
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))


def input_checksum(wl) -> str:
    """sha256 over the raw bytes of the workload's input tensors."""
    import torch
    h = hashlib.sha256()
    for t in (wl.q, wl.k_cache, wl.v_cache, wl.block_tables, wl.context_lens):
        h.update(t.detach().cpu().contiguous().view(torch.uint8).numpy().tobytes())
    return h.hexdigest()


def main(ref_root: str):
    os.environ["TRITON_INTERPRET"] = "1"
    sys.path.insert(0, ref_root)
    sys.path.insert(1, os.path.join(REPO, "coverage-verified-sparse-attention_b200"))
    sys.path.insert(2, REPO)
    import torch
    torch.set_num_threads(os.cpu_count() or 8)
    # reference modules (the checkout's `cvsa` package shadows ours here)
    from cvsa.kernels.page_scores import triton_score_pages
    from cvsa.kernels.sparse_decode import triton_sparse_decode_unnorm
    from cvsa.kernels.coverage import (triton_check_coverage, triton_compute_complement,
                                       triton_lse_merge)
    from cvsa.backend import CVSABackend
    import importlib.util

    def load_local(name, rel):
        spec = importlib.util.spec_from_file_location(name, os.path.join(REPO, rel))
        mod = importlib.util.module_from_spec(spec)
        sys.modules[name] = mod
        spec.loader.exec_module(mod)
        return mod

    synth = load_local("cvsa_synthetic_local",
                       "coverage-verified-sparse-attention_b200/cvsa/synthetic.py")
    oracle = load_local("oracle_cvsa_ref", "oracle/cvsa_ref.py")

    def kernels_case(wl, prefix, out):
        G = wl.num_q_per_kv
        H = wl.num_kv_heads
        bs = wl.block_size
        W = wl.block_tables.shape[1]
        scores = triton_score_pages(wl.q, wl.k_cache, wl.block_tables, wl.context_lens, H, G, bs)
        budget = oracle.budget_for(W, wl.budget_pct)
        idx, nph = oracle.select_pages(scores, wl.context_lens, bs, budget, wl.sink_pages,
                                       wl.local_pages)
        o, m, l = triton_sparse_decode_unnorm(wl.q, wl.k_cache, wl.v_cache, wl.block_tables,
                                              idx, nph, wl.context_lens, H, G, bs)
        acc, cov = triton_check_coverage(scores, idx, nph, wl.tau)
        comp, ncomp = triton_compute_complement(idx, nph, wl.context_lens, bs, acc)
        oc, mc, lc = triton_sparse_decode_unnorm(wl.q, wl.k_cache, wl.v_cache, wl.block_tables,
                                                 comp, ncomp, wl.context_lens, H, G, bs)
        merged = triton_lse_merge(o, m, l, oc, mc, lc, acc, H, G, wl.q.dtype)
        out[prefix + "checksum"] = np.array(input_checksum(wl))
        out[prefix + "scores"] = scores.numpy()
        out[prefix + "sel_idx"] = idx.numpy()
        out[prefix + "sel_n"] = nph.numpy()
        out[prefix + "o_draft"] = o.numpy()
        out[prefix + "m_draft"] = m.numpy()
        out[prefix + "l_draft"] = l.numpy()
        out[prefix + "accept"] = acc.numpy().astype(np.uint8)
        out[prefix + "coverage"] = cov.numpy()
        out[prefix + "n_comp"] = ncomp.numpy()
        out[prefix + "output"] = merged.float().numpy()
        return scores

    out = {}
    # ---- config 1 ----
    wl1 = synth.config1()
    kernels_case(wl1, "config1_", out)
    be = CVSABackend(num_kv_heads=2, num_q_heads=8, head_dim=64, block_size=16,
                     num_layers=1, budget_pct=wl1.budget_pct, coverage_threshold=wl1.tau)
    o_be = be(wl1.q, wl1.k_cache, wl1.v_cache, wl1.block_tables, wl1.context_lens, 0)
    pi, nph = be._cached_selection[0]
    out["config1_backend_output"] = o_be.float().numpy()
    out["config1_backend_sel"] = np.sort(pi[..., :int(nph.max())].numpy(), axis=-1)
    out["config1_backend_n"] = nph.numpy()
    out["config1_backend_accept"] = be._last_accept_mask[0].numpy().astype(np.uint8)

    # ---- small bf16 ragged ----
    wl2 = synth.small(seed=3, B=2, Hq=8, Hkv=2, D=128, ctx=(1000, 2048))
    kernels_case(wl2, "small_", out)
    be = CVSABackend(num_kv_heads=2, num_q_heads=8, head_dim=128, block_size=16,
                     num_layers=1, budget_pct=wl2.budget_pct, coverage_threshold=wl2.tau,
                     lazy=True, check_interval=2)
    g = torch.Generator().manual_seed(11)
    for step in range(5):
        q = torch.randn(wl2.q.shape, generator=g).to(wl2.q.dtype)
        o_s = be(q, wl2.k_cache, wl2.v_cache, wl2.block_tables, wl2.context_lens, 0)
        be.step_done(0, 1)
        out[f"small_lazy_q{step}"] = q.float().numpy()
        out[f"small_lazy_out{step}"] = o_s.float().numpy()
    st = be.get_stats()
    for key in ("total_scoring_steps", "total_coverage_checks", "all_accepted_pct",
                "some_rejected_pct", "per_head_accept_rate", "effective_budget_pct"):
        out["small_lazy_stat_" + key] = np.array(st[key], dtype=np.float64)

    path = os.path.join(HERE, "reference_outputs.npz")
    np.savez_compressed(path, **out)
    print("wrote", path, os.path.getsize(path), "bytes")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit(f"usage: python {sys.argv[0]} <path to the reference checkout>")
    main(sys.argv[1])
