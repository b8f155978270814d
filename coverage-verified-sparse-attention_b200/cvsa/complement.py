"""Complement page set (drop-in for cvsa/complement.py:11-69), on the GPU.

Same signature and result as the reference's sort-based PyTorch version
(indices of valid pages not selected, n = 0 for accepted heads); the list is
in ascending page order and its width is the largest complement, like the
reference (a [B, H_kv, 1] zero tensor when every complement is empty).
"""

from typing import Tuple

import torch

from cvsa.kernels.coverage import compute_complement


def compute_complement_pages(page_indices: torch.Tensor, n_per_head: torch.Tensor,
                             context_lens: torch.Tensor, block_size: int,
                             accept_mask: torch.Tensor = None
                             ) -> Tuple[torch.Tensor, torch.Tensor]:
    comp, n_comp = compute_complement(page_indices, n_per_head, context_lens, block_size,
                                      accept_mask)
    max_c = int(n_comp.max().item()) if n_comp.numel() else 0   # complement.py:60 syncs too
    if max_c == 0:
        B, H = n_per_head.shape
        return torch.zeros((B, H, 1), dtype=torch.int32, device=comp.device), n_comp
    return comp[:, :, :max_c].contiguous(), n_comp
