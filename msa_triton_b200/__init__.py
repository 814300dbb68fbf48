"""B200-native (sm_100a) MiniMax-M3 three-stage sparse attention.

Drop-in for the operators of yeyeyeping/msa_triton (``msa_triton.triton``):

    scores  = m3_index_score(index_q, index_k, cu_seqlens, max_seqlen, block_size=128, scale=1.0)
    indices = m3_topk(scores, cu_seqlens, block_size=128, topk_blocks=16, local_blocks=1)
    out     = m3_sparse_attention(q, k, v, indices, cu_seqlens, max_seqlen, block_size=128)

plus the indexer's KL objective on the selected tokens, which the reference
specifies without implementing it (``m3_index_kl_loss``), and the three stages
for decode over a paged KV cache (``m3_index_score_decode``, ``m3_topk_decode``,
``m3_sparse_decode``).

Same signatures, TND layout, int32 ``cu_seqlens`` and autograd behaviour (plus
an optional ``prepared=prepare_batch(cu_seqlens)`` keyword that reads the
boundaries to the host once for every op and layer that shares them); the
work runs in hand-written CUDA kernels (``libmsa_b200.so``, C ABI in
``include/msa_b200.h``). Importing the package does not load the library.
"""

from .decode import m3_index_score_decode, m3_sparse_decode, m3_topk_decode
from .index_kl import m3_index_kl_loss
from .index_score import m3_index_score
from .prepared import PreparedBatch, prepare_batch
from .sparse_attention import m3_sparse_attention
from .topk import m3_topk

__all__ = ["m3_index_score", "m3_topk", "m3_sparse_attention", "m3_index_kl_loss", "m3_index_score_decode",
           "m3_topk_decode", "m3_sparse_decode", "prepare_batch", "PreparedBatch"]
