"""TEST INFRASTRUCTURE ONLY — CPU oracle for the packed-KV hot path.

A restatement, in this project's own code, of the reference's CPU algorithm
(zoaibs/Dynamic-KV-Cache):

  kvq.py      numpy restatement of the groupwise quantiser and its 'DKVC'
              header (src/kv_quantization.py:12-92) — bit-exact byte/integer work.
  cpu_path.py torch-CPU restatement of the reference's CPU cache path
              (src/cache_manager.py:43-63: unpack history, keep the current frame
              native, then SDPA with the bottom-right causal mask of
              tests/test_gpu_backend.py:97-100) — the attention oracle and the
              timed CPU baseline ("port").
  pools.py    host model of the GPU pool layout (src/gpu_cache.py:36-41) so GPU
              pools can be compared byte for byte with kvq.pack output.
  decoder.py  plain-torch restatement of the SmolLM2-360M-shape decoder path with
              the mixed-precision cache semantics and the candidate
              log-likelihood protocol (src/streaming.py:209-225).

Parity is pinned: tests/test_oracle_golden.py checks this oracle against golden
vectors produced by the reference itself (its CPU quantiser and its Triton
kernels run in the Triton interpreter; tests/golden/make_golden.py).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference
legs may import this package. The product (dynamic-kv-cache_b200/) never does.
"""
