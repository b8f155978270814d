"""Top-k page selection from page scores (replaces cvsa/backend.py:737-747).

The reference calls torch.topk(sorted=False) and clamps n_per_head to
min(budget, n_valid). Here selection runs on the GPU (csrc/select.cu) with a
defined order -- (score desc, page index asc), so ties go to the lower page
index -- an optional set of always-kept sink/local pages, and the result in
ascending page order.
"""

from typing import Tuple

import torch

from cvsa import _lib


def budget_for(table_width: int, budget_pct: float) -> int:
    """cvsa/backend.py:690: max(3, int(max_pages * budget_pct))."""
    return max(3, int(table_width * budget_pct))


def select_pages(page_scores: torch.Tensor, context_lens: torch.Tensor, block_size: int,
                 budget: int, sink_pages: int = 0, local_pages: int = 0,
                 max_sel: int = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """(page_indices [B, H_kv, max_sel] int32 ascending, n_per_head [B, H_kv] int32)."""
    dev = _lib.require_cuda(page_scores, context_lens)
    B, H, W = page_scores.shape
    if max_sel is None:
        max_sel = budget + sink_pages + local_pages
    ps = page_scores.float().contiguous()
    idx = torch.zeros((B, H, max(max_sel, 1)), dtype=torch.int32, device=dev)
    n = torch.zeros((B, H), dtype=torch.int32, device=dev)
    lib = _lib.load()
    _lib.check(lib.cvsa_select_pages(ps.data_ptr(), B, H, W, context_lens.data_ptr(), block_size,
                                     budget, sink_pages, local_pages, idx.data_ptr(),
                                     max(max_sel, 1), n.data_ptr(), _lib.stream_ptr(dev)),
               "cvsa_select_pages")
    return idx, n
