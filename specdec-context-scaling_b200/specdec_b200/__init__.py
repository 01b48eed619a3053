"""specdec_b200 -- B200-native decode-side attention path of the Qwen2.5 greedy
speculative-decoding engine (RichardF123/SpecDec-Context-Scaling).

Subpackages:
  kernels  -- ops / patch / build, the drop-in for specdec/kernels
  engine   -- paged KV cache, spec_cache contract, batched SpecDec engine
"""

__version__ = "0.1.0"
