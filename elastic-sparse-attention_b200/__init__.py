"""B200-native elastic sparse attention (sm_100a CUDA kernels behind a C ABI).

Drop-in for ``elastic_sparse_attention.ElasticSparseAttention`` of
HighCWu/elastic-sparse-attention.  Import it as ``elastic_sparse_attention_b200``
(the loader module of that name at the repository root maps it to this
directory).
"""
from . import _lib, layer_ops, ops
from .attention import ElasticSparseAttention, ElasticSparseAttentionFunction, KeyPlanCache
from .decoder import ElasticDecoderStack
from .head_split import HeadShardedElasticSparseAttention, head_share
from .ops import PatternSpec
from .sharded import SequenceShardedElasticSparseAttention

__all__ = ["ElasticSparseAttention", "ElasticSparseAttentionFunction", "ElasticDecoderStack",
           "HeadShardedElasticSparseAttention", "KeyPlanCache", "PatternSpec",
           "SequenceShardedElasticSparseAttention", "head_share", "layer_ops", "ops", "_lib"]
__version__ = "0.1.3"
