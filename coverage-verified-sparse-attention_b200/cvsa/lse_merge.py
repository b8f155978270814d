"""Selective LSE merge (drop-in for cvsa/lse_merge.py:11-54), on the GPU."""

import torch

from cvsa.kernels.coverage import lse_merge


def selective_lse_merge(o_draft, m_draft, l_draft, o_comp, m_comp, l_comp, accept_mask,
                        num_q_per_kv: int, output_dtype: torch.dtype = torch.bfloat16
                        ) -> torch.Tensor:
    num_kv_heads = accept_mask.shape[1]
    return lse_merge(o_draft, m_draft, l_draft, o_comp, m_comp, l_comp, accept_mask,
                     num_kv_heads, num_q_per_kv, output_dtype)
