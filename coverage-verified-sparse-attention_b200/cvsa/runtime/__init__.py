"""Paged KV store and dense-layer attention on the B200 kernels."""
