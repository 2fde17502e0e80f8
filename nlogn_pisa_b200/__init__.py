"""B200 (sm_100a) implementation of PISA's hot path: hierarchical LSE block
selection over a mean-pooled key pyramid, then attention over the selected
key blocks.

The operators keep the reference package's names and signatures
(``pisa.ops``: select_blocks / top_k_pyramid_fn, sparse_attention /
sparse_attn_fn, mean_pool, build_pyramid; ``xmixers`` PyramidCache /
TensorCache).  All computation runs in the hand-written CUDA library
``libpisa_b200.so`` through its C ABI (include/pisa_b200.h).
"""

from .attention import sparse_attention, sparse_attn_fn
from .cache import PyramidCache, TensorCache
from ._lib import set_status_checks
from .selection import (bsa_fn, build_pyramid, decode_select_attend, grouped_leaf_scores, mean_pool,
                        routing_geometry, select_blocks, top_k_pyramid_fn)

mean_pooling_fn = mean_pool

__all__ = [
    "select_blocks", "top_k_pyramid_fn", "sparse_attention", "sparse_attn_fn", "mean_pool",
    "mean_pooling_fn", "build_pyramid", "routing_geometry", "PyramidCache", "TensorCache",
    "grouped_leaf_scores", "set_status_checks", "decode_select_attend", "bsa_fn",
]
