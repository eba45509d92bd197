"""tsb: the B200-native verify-pass hot path of mlx-tree-spec.

Operators (reference-facing, over torch CUDA tensors):
  quantized_matmul, dequantize, ancestor_bits, tree_flash, mask_bits, sdpa
Containers: KVCache, Q8KVCache, MLXQ8KVCache
Input makers: quantize, quantize_rows, quantize_g64
Sharding: tsb.dist (N-sharded qmm: GatheredQMM gathers the output inside the
  kernel over NVLink; ShardedQMM uses an NCCL all-gather)
Decoder: tsb.decoder (the verify-step layer stack over the qmm, tree attention
  and the decoder-layer kernels)
Tree commit: keep_kv, commit (keep the accepted path's K/V rows)
Checkpoints: tsb.checkpoint (mlx-lm safetensors -> device buffers, per-rank
  row shards, fused q|k|v and gate|up)
GatedDeltaNet: tsb.gdn (the hybrid model's linear-attention layers over tree
  nodes: gdn_prep, tree_gated_delta, gdn_commit)

All compute runs in libtsb.so (sm_100a CUDA); importing the operators loads
it and fails loudly if it is missing.
"""

from . import _lib
from ._lib import (TSB_KV_BF16, TSB_KV_MLX_Q8_G64, TSB_KV_REF_Q8_ROW, TSBError,  # noqa: F401
                   load as load_library)
from .cache import KVCache, MLXQ8KVCache, Q8KVCache  # noqa: F401
from .ops import (ancestor_bits, commit, dequantize, keep_kv, mask_bits, quantized_matmul, sdpa,  # noqa: F401
                  tree_flash, workspace)
from .quant import quantize, quantize_g64, quantize_rows  # noqa: F401

__version__ = "0.1.0"
