"""B200-native (sm_100a) splitzip KV codec: the UnchainKV KV-transfer hot path.

Modules:
  splitzip_cuda  operator API of the codec (mirror of unchain_kv.splitzip_cuda),
                 plus the batched, device-chosen codec, attention, calibration
                 and writeback entry points
  tensor_blocks  byte chunking of block payloads
  transport      GPU-to-GPU stream transport (decode straight from a peer)
  workloads      seeded synthetic KV caches and palettes of the benchmark configs
  _build         nvcc build of the sm_100a C-ABI library
"""

__version__ = "0.1.0"
