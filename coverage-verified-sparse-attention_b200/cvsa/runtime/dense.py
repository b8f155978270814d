"""Dense paged decode for dense layers (drop-in for cvsa/runtime/dense.py).

The reference calls FlashInfer's BatchDecodeWithPagedKVCacheWrapper with a
Triton fallback (dense.py:70-111). Here a dense layer is the same split-K
GQA-packed decode kernel run over every valid page (cvsa_decode_step in
CVSA_MODE_DENSE); there is no library or fallback path.
"""

import torch

from cvsa import _lib


class DenseAttentionBackend:
    def __init__(self, num_kv_heads, num_q_heads, head_dim, block_size):
        self.num_kv_heads = num_kv_heads
        self.num_q_heads = num_q_heads
        self.num_q_per_kv = num_q_heads // num_kv_heads
        self.head_dim = head_dim
        self.block_size = block_size
        self._idx = {}

    def reset(self):
        pass

    def step_done(self, layer_idx, num_layers):
        pass

    def __call__(self, q, k_cache, v_cache, block_tables, context_lens, layer_idx=0):
        """q: [B, H_q, D] -> [B, H_q, D] in q's dtype."""
        dev = _lib.require_cuda(q, k_cache, v_cache, block_tables, context_lens)
        q = q.contiguous()
        B = q.shape[0]
        bt = block_tables.to(torch.int32).contiguous()
        cl = context_lens.to(torch.int32).contiguous()
        out = torch.empty_like(q)
        key = (dev, B)
        dummy = self._idx.get(key)
        if dummy is None:
            dummy = (torch.zeros((B, self.num_kv_heads, 1), dtype=torch.int32, device=dev),
                     torch.zeros((B, self.num_kv_heads), dtype=torch.int32, device=dev))
            self._idx[key] = dummy
        kvd = _lib.kv_desc(k_cache, v_cache)
        qd = _lib.query_desc(q, bt, cl)
        cfg = _lib.StepConfig(_lib.MODE_DENSE, 0, 0, 0, 0.0, _lib.RECOVERY_EXACT, 0, 0)
        io = _lib.StepIO(dummy[0].data_ptr(), dummy[1].data_ptr(), 1, 0, out.data_ptr(), None,
                         None, None, None, None, None)
        lib = _lib.load()
        nbytes = lib.cvsa_step_workspace_size(qd, kvd, cfg, 1)
        ws = _lib.WORKSPACE.get(nbytes, dev, "step")
        _lib.check(lib.cvsa_decode_step(qd, kvd, cfg, io, ws.data_ptr(), ws.numel(),
                                        _lib.stream_ptr(dev)), "cvsa_decode_step(dense)")
        return out
