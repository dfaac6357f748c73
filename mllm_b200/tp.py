"""Tensor-parallel attention across GPUs: KV-head-group sharding + one o_proj all-reduce.

The reference runs every layer on one device (QwenRunner.cpp:236,328); across N GPUs the
attention path shards naturally by KV-head group:

  rank r owns kv heads [r*Hkv/N, (r+1)*Hkv/N) and their n_rep query heads each, so
    w_q / w_k / w_v   row slices   (the projections of the owned heads)
    QK-norm, RoPE, KV cache, prefill / decode attention   fully local
    w_o               column slice (o_proj of the owned heads' outputs) -> a partial [B, S, hidden]
  and the partial outputs are summed by ONE all-reduce (NCCL over NVLink on GPUs).

`attention_fn` computes the local attention block; the default is the B200 path
(mllm_b200.runtime.attention_block).  The all-reduce uses the given torch.distributed group.
"""
from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True)
class HeadShard:
    rank: int
    world: int
    q_heads: tuple   # [start, end)
    kv_heads: tuple  # [start, end)

    @property
    def num_heads(self) -> int:
        return self.q_heads[1] - self.q_heads[0]

    @property
    def num_kv_heads(self) -> int:
        return self.kv_heads[1] - self.kv_heads[0]


def shard_heads(num_heads: int, num_kv_heads: int, world: int, rank: int) -> HeadShard:
    """KV-head groups split evenly over `world` ranks (num_kv_heads % world == 0)."""
    if num_heads % num_kv_heads != 0:
        raise RuntimeError("Attention: num_heads must be divisible by num_kv_heads.")
    if num_kv_heads % world != 0:
        raise RuntimeError(f"tensor parallel: {num_kv_heads} kv heads do not split over {world} ranks")
    if not 0 <= rank < world:
        raise RuntimeError("tensor parallel: rank out of range")
    n_rep = num_heads // num_kv_heads
    per = num_kv_heads // world
    g0, g1 = rank * per, (rank + 1) * per
    return HeadShard(rank, world, (g0 * n_rep, g1 * n_rep), (g0, g1))


def shard_weights(shard: HeadShard, head_dim: int, w_q, w_k, w_v, w_o):
    """Row slices of w_q/w_k/w_v ([out, in], HF layout) and the column slice of w_o."""
    q0, q1 = shard.q_heads[0] * head_dim, shard.q_heads[1] * head_dim
    k0, k1 = shard.kv_heads[0] * head_dim, shard.kv_heads[1] * head_dim
    return (w_q[q0:q1].contiguous(), w_k[k0:k1].contiguous(), w_v[k0:k1].contiguous(),
            w_o[:, q0:q1].contiguous())


def tp_attention_block(h, shard: HeadShard, head_dim: int, rope_theta: float, position_ids, kv_cache,
                       w_q, w_k, w_v, w_o, w_q_norm=None, w_k_norm=None, rms_norm_eps: float = 1e-6,
                       group=None, attention_fn=None):
    """The attention half of TransformerBlock::Forward on this rank's heads, then the o_proj
    all-reduce.  Weights are this rank's slices (shard_weights); kv_cache holds only the owned
    kv heads.  Returns the full [B, S, hidden] attention output on every rank."""
    import torch.distributed as dist
    if attention_fn is None:
        from .runtime import attention_block as attention_fn
    partial = attention_fn(h, w_q, w_k, w_v, w_o, shard.num_heads, shard.num_kv_heads, head_dim, rope_theta,
                           position_ids, kv_cache, w_q_norm, w_k_norm, rms_norm_eps)
    if shard.world > 1:
        dist.all_reduce(partial, op=dist.ReduceOp.SUM, group=group)
    return partial
