"""nanoslg_b200: B200-native (sm_100a) kernels behind NanoSLG's per-layer attention path.

Modules mirror the reference's interfaces for this path:
  kv_cache   -- CacheContext / KVCacheManager ABCs, page pool, radix tree, B200 context
  models     -- Llama TP / PP / hybrid models calling the context per layer
  tp_layers  -- Column/RowParallelLinear, ParallelLMHead
  parallel   -- ParallelConfig / ParallelContext and the TP collectives
  ops        -- torch wrappers of the C ABI (include/nslg_b200.h)
  build      -- nvcc build of nanoslg_b200/lib/libnslg_b200.so
"""
__version__ = "0.1.0"
