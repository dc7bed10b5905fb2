"""CPU oracle for nano-vLLM's attention hot path — TEST INFRASTRUCTURE ONLY.

This package restates, in numpy, the arithmetic of the path that the B200
kernels replace, so that tests can check the CUDA results on the same seeded
inputs.  Only `tests/`, `__graft_entry__.smoke()` and the CPU-baseline leg of
`bench.py` may import it, and only as the checker or as the timed CPU
baseline.  The product path (`learn-nano-vllm_b200`) never imports it and has
no CPU fallback.

Modules
  kv_store      slot-mapped KV-cache scatter  (nanovllm/layers/attention.py:10-40)
  attention     paged decode / verify attention and causal varlen prefill
                (the flash-attn calls of nanovllm/layers/attention.py:64-74)
  spec_sampling speculative acceptance sampling with the fixed-order
                arithmetic the CUDA kernel uses
  cases         seeded case factories for the benchmark configurations

Pinning
  * kv_store is pinned bit-exactly to the reference's own Triton kernel run
    under TRITON_INTERPRET=1 (fixtures in tests/golden/, generator script
    beside them) and to the store contract's hand-worked example in the
    reference's study guide (master_nano-vllm-v2.md:2830-2852).
  * attention is pinned to outputs of flash-attn 2.8.3 — the library the
    reference calls at nanovllm/layers/attention.py:67-74 — run on a B200 on
    the same seeded inputs (fixtures in tests/golden/, generator beside them).
  * spec_sampling restates the standard rejection scheme; the reference has
    no speculative path, so it has nothing to be pinned against.
"""
