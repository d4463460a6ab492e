"""B200-native (sm_100a) SmoothQuant W8A8 linear and vocab-sharded LM head.

The compute path is libw8a8.so (hand-written CUDA kernels behind the C ABI in
include/w8a8.h); this package is its host-side mirror of romanaccio's operator surface.
"""
from ._lib import (ACT_DYNTOK, ACT_STATIC, DTYPE_FP16, DTYPE_INT8, DTYPE_INT16, OUT_ACC_I32,
                   OUT_F32, OUT_F32_ACC, OUT_QUANT, PATH_AUTO, PATH_GEMV, PATH_TENSOR, TOPK_MAX,
                   W8A8Error)
from .linear import Context, Linear16, SubgraphScaleInfo, W8A8Linear, topk_merge
from .lmhead import (LmHeadShard, MultiDeviceLmHead, RankLmHead, VocabShardedLmHead,
                     shard_range)
from .norm import emb_norm_pack, emb_norm_scaled, post_op_ffn_pack, rmsnorm_pack_dyntok
from .package import load_quant_scales, read_weight_region, untile_int8, untile_int16
from .sampler import CandidateSampler, SamplingConfig

__all__ = [
    "ACT_DYNTOK", "ACT_STATIC", "DTYPE_FP16", "DTYPE_INT8", "DTYPE_INT16", "OUT_ACC_I32",
    "OUT_F32", "OUT_F32_ACC", "OUT_QUANT", "PATH_AUTO", "PATH_GEMV", "PATH_TENSOR", "TOPK_MAX",
    "W8A8Error", "Context",
    "SubgraphScaleInfo", "W8A8Linear", "Linear16", "topk_merge", "LmHeadShard", "MultiDeviceLmHead",
    "RankLmHead",
    "VocabShardedLmHead",
    "shard_range", "CandidateSampler", "SamplingConfig", "rmsnorm_pack_dyntok",
    "post_op_ffn_pack", "emb_norm_pack", "emb_norm_scaled", "load_quant_scales", "read_weight_region", "untile_int8", "untile_int16",
]
