"""CPU oracle of the decode-attention path -- TEST INFRASTRUCTURE ONLY.

This package restates, on the CPU, the reference algorithms the CUDA path
replaces (RichardF123/SpecDec-Context-Scaling):

  attention.py  reference.attention / attention_fp32   (specdec/kernels/reference.py:33-70)
  fp8.py        quantize_kv_fp8 / dequantize_kv_fp8     (specdec/engine/model_self.py:300-320)
                and torch's float8_e4m3fn rounding       (c10 Float8_e4m3fn, RNE, NaN above 464)
  paged.py      the paged pool layout of specdec_b200 and its gather back to (B, KV, T, D)
  spec_cache.py cache_length / trim_cache / check_consistent (specdec/engine/spec_cache.py:4-46)
  accept.py     greedy accept, strict and vectorised     (spec_dec.py:230-250,
                                                          fast_spec_dec.py:246-256)
  engine.py     a small Qwen2 decoder with the reference cache semantics (model_self.py:668-931)
  elementwise.py reference.rmsnorm / apply_rope / swiglu  (specdec/kernels/reference.py:14-31)
  specdec.py    the strict greedy SpecDec executor       (specdec/engine/spec_dec.py:189-275)

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import
it, always as the checker or the timed CPU baseline; the product path
(specdec_b200) never imports it.  It is pinned against golden vectors
produced by the live reference (tests/golden/make_golden.py).
"""
