"""B200-native (sm_100a) splitzip KV codec: the UnchainKV KV-transfer hot path.

Modules:
  splitzip_cuda  operator API of the codec (mirror of unchain_kv.splitzip_cuda)
  codec          connector-level producer/receiver dispatch (mode fallback chain)
  tensor_blocks  byte chunking of block payloads
  workloads      seeded synthetic KV caches and palettes of the benchmark configs
"""

__version__ = "0.1.0"
