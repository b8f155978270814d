"""Golden fixture for the paged KV runtime, from the REFERENCE.

Run once, in a container that has the reference checkout (not on the GPU box):

    python tests/golden/make_golden_kv.py /path/to/coverage-verified-sparse-attention

It runs the reference's PagedKVCache and SequenceKVManager
(cvsa/runtime/kv_cache.py) on CPU tensors through a seeded schedule
(`schedule()`, shared with the tests): three sequences prefilled with 37,
16 and 70 tokens, then 40 decode steps appending one token to each sequence
in turn (pages fill, new blocks are taken from the bump allocator). Stored:
the block tables, context lengths, pages allocated and the next free block
after the prefills and at the end, and sha256 digests of the K and V pools.
"""

from __future__ import annotations

import hashlib
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))

NUM_BLOCKS, BS, H, D, B, MAX_CTX = 24, 16, 2, 64, 3, 160
PREFILL = (37, 16, 70)
STEPS = 40


def schedule():
    """(prefills: list of (seq, k, v)), (appends: list of (seq, k, v)), bf16 CPU."""
    import torch
    g = torch.Generator().manual_seed(77)
    pre = []
    for b, n in enumerate(PREFILL):
        k = torch.randn((n, H, D), generator=g).to(torch.bfloat16)
        v = torch.randn((n, H, D), generator=g).to(torch.bfloat16)
        pre.append((b, k, v))
    app = []
    for s in range(STEPS):
        b = s % B
        k = torch.randn((H, D), generator=g).to(torch.bfloat16)
        v = torch.randn((H, D), generator=g).to(torch.bfloat16)
        app.append((b, k, v))
    return pre, app


def digest(t) -> str:
    return hashlib.sha256(t.contiguous().view(-1).view(__import__("torch").uint8)
                          .numpy().tobytes()).hexdigest()


def main(ref_root: str):
    sys.path.insert(0, ref_root)
    import torch
    from cvsa.runtime.kv_cache import PagedKVCache, SequenceKVManager   # the reference's
    cache = PagedKVCache(NUM_BLOCKS, BS, H, D, dtype=torch.bfloat16, device="cpu")
    mgr = SequenceKVManager(cache, B, MAX_CTX)
    pre, app = schedule()
    out = {}
    for b, k, v in pre:
        mgr.prefill_kv(b, k, v)
    out["pre_tables"] = mgr.block_tables.numpy().copy()
    out["pre_lens"] = mgr.context_lens.numpy().copy()
    out["pre_pages"] = np.array(mgr._pages_allocated, dtype=np.int32)
    out["pre_next_free"] = np.array(cache._next_free)
    for b, k, v in app:
        mgr.append_token_kv(b, k, v)
    out["tables"] = mgr.block_tables.numpy()
    out["lens"] = mgr.context_lens.numpy()
    out["pages"] = np.array(mgr._pages_allocated, dtype=np.int32)
    out["next_free"] = np.array(cache._next_free)
    out["k_sha"] = np.array(digest(cache.k_cache))
    out["v_sha"] = np.array(digest(cache.v_cache))
    path = os.path.join(HERE, "reference_outputs_kv.npz")
    np.savez_compressed(path, **out)
    print("wrote", path, os.path.getsize(path), "bytes")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit(f"usage: python {sys.argv[0]} <path to the reference checkout>")
    main(sys.argv[1])
