"""Vocabulary-parallel grammar-conditioned LM head (one process per GPU).

The reference is single-GPU. A large-vocabulary head shards naturally by
vocabulary rows: rank r owns the contiguous rows [start_r, stop_r) of W and
the matching words of every request's bitmask (shard boundaries are multiples
of 32 tokens, so a shard owns whole mask words), runs the same kernels on its
slice with vocab_offset = start_r, and the ranks exchange only

  * one signed-orderable int64 top-1 key per request (an integer MAX
    all-reduce: the larger rounded logit wins, ties go to the lower global
    token id), decoded on the device by gsp_top1_from_keys; and
  * when full logits are requested, the -inf-filled [B, V/R] logit slices
    (an all-gather).

Two ways to merge the top-1: `PeerExchange` (the default on GPUs) does it
inside the projection kernel - the last CTA of every rank stores its keys
into every rank's exchange buffer over NVLink and waits for the others'
(gsp_vocab_parallel_logits), so a step is one launch and no collective;
without one, keys go through a torch.distributed MAX all-reduce (NCCL between
GPUs; gloo works for the host-side logic on CPU ranks) and a decode launch.
Full logits always go through an all-gather.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from . import _native

KEY_SIGN = -(1 << 63)  # XOR with this flips the top bit of an int64


class ExchangeTimeout(RuntimeError):
    """A rank's in-kernel wait for the other ranks' top-1 keys ran out (a peer
    stalled or left): the call reported no token (top_index -1). The group
    must call PeerExchange.reset() on every rank before its next call."""


def check_exchange(top_index: torch.Tensor) -> None:
    """Raises ExchangeTimeout when a vocabulary-parallel call reported no
    token (top_index -1, the in-kernel exchange's time-out marker). Reads the
    tensor on the host: call it where the step's result is read anyway."""
    if bool((top_index < 0).any()):
        raise ExchangeTimeout("the cross-rank top-1 exchange timed out; call PeerExchange.reset() on every rank")


def shard_bounds(vocab: int, world_size: int, rank: int, align: int = 32) -> tuple[int, int]:
    """Contiguous row range of `rank`: boundaries are multiples of `align`
    (whole mask words), sizes differ by at most one `align` block, the last
    shard takes the ragged tail."""
    if world_size < 1 or not 0 <= rank < world_size:
        raise ValueError("bad rank / world size")
    blocks = (vocab + align - 1) // align
    lo_blk = blocks * rank // world_size
    hi_blk = blocks * (rank + 1) // world_size
    return min(lo_blk * align, vocab), min(hi_blk * align, vocab)


# ---------------------------------------------------------------------------
# top-1 keys (host mirror of the device packing in csrc/gsp_common.cuh)
# ---------------------------------------------------------------------------
def _ordered_bits(values: torch.Tensor) -> torch.Tensor:
    v = values.to(torch.float32).clone()
    v[v == 0] = 0.0  # +0 and -0 compare equal
    u = v.view(torch.int32).to(torch.int64) & 0xFFFFFFFF
    neg = (u & 0x80000000) != 0
    return torch.where(neg, (~u) & 0xFFFFFFFF, u | 0x80000000)


def encode_keys(rounded_values: torch.Tensor, global_index: torch.Tensor, valid: torch.Tensor | None = None) -> torch.Tensor:
    """Signed-orderable int64 keys of (rounded logit, global token id); rows
    with no legal token (valid False) get the empty key."""
    hi = _ordered_bits(rounded_values)
    lo = 0xFFFFFFFF - (global_index.to(torch.int64) & 0xFFFFFFFF)
    unsigned = (hi << 32) | lo  # wraps into the sign bit exactly like uint64
    keys = unsigned ^ KEY_SIGN
    if valid is not None:
        keys = torch.where(valid, keys, torch.full_like(keys, KEY_SIGN))
    return keys


def decode_keys(keys: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """int64 keys -> (float32 value, int64 token id); the empty key decodes to
    (-inf, 0), as torch.argmax of an all -inf row."""
    unsigned = keys.to(torch.int64) ^ KEY_SIGN
    empty = unsigned == 0
    hi = (unsigned >> 32) & 0xFFFFFFFF
    lo = unsigned & 0xFFFFFFFF
    bits = torch.where((hi & 0x80000000) != 0, hi & 0x7FFFFFFF, (~hi) & 0xFFFFFFFF)
    vals = bits.to(torch.int32).view(torch.float32) if bits.numel() else bits.to(torch.float32)
    vals = torch.where(empty, torch.full_like(vals, float("-inf")), vals)
    idx = torch.where(empty, torch.zeros_like(lo), 0xFFFFFFFF - lo)
    return vals, idx


def merge_top1_keys(keys: torch.Tensor, group=None) -> torch.Tensor:
    """In-place integer MAX all-reduce of per-request keys across the ranks."""
    if dist.is_initialized() and dist.get_world_size(group) > 1:
        dist.all_reduce(keys, op=dist.ReduceOp.MAX, group=group)
    return keys


def gather_logits(local: torch.Tensor, vocab: int, group=None) -> torch.Tensor:
    """All-gather [B, V_r] logit slices into [B, V] (ranks in order). Slices
    are padded to the largest shard for the collective."""
    if not (dist.is_initialized() and dist.get_world_size(group) > 1):
        return local
    world = dist.get_world_size(group)
    bounds = [shard_bounds(vocab, world, r) for r in range(world)]
    width = max(hi - lo for lo, hi in bounds)
    batch = local.shape[0]
    padded = torch.full((batch, width), float("-inf"), dtype=local.dtype, device=local.device)
    padded[:, : local.shape[1]] = local
    parts = [torch.empty_like(padded) for _ in range(world)]
    dist.all_gather(parts, padded.contiguous(), group=group)
    return torch.cat([p[:, : hi - lo] for p, (lo, hi) in zip(parts, bounds)], dim=1)


class PeerExchange:
    """Exchange buffers of a vocabulary-parallel group for the in-kernel top-1
    merge: this rank's own buffer plus every other rank's, mapped into this
    process through CUDA IPC (one node). Creating and closing are collective:
    every rank of `group` must take part, in the same order."""

    def __init__(self, max_batch: int, group=None, wait_us: int = 250_000):
        if not dist.is_initialized():
            raise RuntimeError("PeerExchange needs an initialised process group")
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > _native.MAX_PEERS:
            raise ValueError(f"at most {_native.MAX_PEERS} ranks share an exchange")
        self.max_batch = int(max_batch)
        self.wait_us = int(wait_us)  # longest in-kernel wait for the other ranks' keys
        self.group = group
        self.own, handle = _native.peer_exchange_alloc(self.world, self.max_batch)
        handles = [None] * self.world
        dist.all_gather_object(handles, handle, group=group)
        self.peers = [self.own if q == self.rank else _native.peer_exchange_open(h) for q, h in enumerate(handles)]
        dist.barrier(group)  # every rank has mapped every buffer before any kernel writes

    def reset(self) -> None:
        """Collective re-synchronisation after a wait ran out (ExchangeTimeout):
        every rank waits for its own calls, the group meets at a barrier, each
        rank zeroes its own buffer (epoch, flags, keys) and its workspace, and
        the group meets again before anyone calls the exchange."""
        torch.cuda.synchronize()
        dist.barrier(self.group)
        _native.peer_exchange_reset(self.own, self.world, self.max_batch)
        _native.reset_workspace(torch.device("cuda", torch.cuda.current_device()))
        torch.cuda.synchronize()
        dist.barrier(self.group)

    def close(self) -> None:
        """Collective: after every rank's last exchange call has completed."""
        if self.own is None:
            return
        torch.cuda.synchronize()
        dist.barrier(self.group)
        for q, ptr in enumerate(self.peers):
            if q != self.rank:
                _native.peer_exchange_close(ptr)
        dist.barrier(self.group)
        _native.peer_exchange_free(self.own)
        self.own = None
        self.peers = []


class VocabParallelHead:
    """This rank's shard of a vocabulary-parallel LM head.

    forward(hidden [B, H], bitmask_gpu [B, >= ceil(V/32)] full-vocabulary
    mask) -> (top_value [B] float32, top_index [B] int64 global ids,
    logits [B, V] or None). Every rank must call forward with the same
    arguments in the same order (the collectives are matched by order).
    """

    def __init__(self, weight_shard: torch.Tensor, vocab: int, start: int, group=None,
                 exchange: PeerExchange | None = None):
        if weight_shard.device.type != "cuda":
            raise ValueError("weight_shard must be a CUDA tensor")
        if start % 32:
            raise ValueError("shard start must be a multiple of 32")
        self.weight = weight_shard.contiguous()
        self.vocab = vocab
        self.start = start
        self.stop = start + weight_shard.shape[0]
        self.group = group
        self.exchange = exchange
        if exchange is not None and self.stop <= self.start:
            raise ValueError("every rank of a peer exchange needs a non-empty shard")

    @classmethod
    def from_full_weight(cls, weight: torch.Tensor, group=None,
                         exchange: PeerExchange | None = None) -> "VocabParallelHead":
        world = dist.get_world_size(group) if dist.is_initialized() else 1
        rank = dist.get_rank(group) if dist.is_initialized() else 0
        lo, hi = shard_bounds(weight.shape[0], world, rank)
        return cls(weight[lo:hi], weight.shape[0], lo, group, exchange)

    def local_mask(self, bitmask_gpu: torch.Tensor) -> torch.Tensor:
        w0 = self.start // 32
        w1 = (self.stop + 31) // 32
        return bitmask_gpu[:, w0:w1]

    def forward(self, hidden: torch.Tensor, bitmask_gpu: torch.Tensor | None, *,
                route: str = "row-sparse", full_logits: bool = False, check: bool = True):
        """With the peer exchange, check=True reads top_index back and raises
        ExchangeTimeout when the in-kernel wait ran out (no partial merge is
        ever returned as a token); check=False leaves that to the caller
        (check_exchange), e.g. under CUDA-graph capture."""
        hidden_2d = hidden.reshape(1, -1) if hidden.ndim == 1 else hidden
        batch = hidden_2d.shape[0]
        dev = hidden.device
        mask = None if bitmask_gpu is None else self.local_mask(bitmask_gpu.reshape(batch, -1))
        local_logits = (torch.empty((batch, self.stop - self.start), device=dev, dtype=hidden.dtype)
                        if full_logits else None)
        if self.exchange is not None:
            top_value = torch.empty(batch, device=dev, dtype=torch.float32)
            top_index = torch.empty(batch, device=dev, dtype=torch.int64)
            _native.vocab_parallel(route, hidden_2d, self.weight, mask, self.exchange.peers, self.exchange.rank,
                                   self.exchange.max_batch, self.vocab, logits=local_logits,
                                   top_value=top_value, top_index=top_index, vocab_offset=self.start,
                                   wait_us=self.exchange.wait_us)
            if check:
                check_exchange(top_index)
            logits = gather_logits(local_logits, self.vocab, self.group) if full_logits else None
            return top_value, top_index, logits
        keys = torch.empty(batch, device=dev, dtype=torch.int64)
        fn = {"row-sparse": _native.row_sparse, "block-sparse": _native.block_gemm,
              "dense-mask": _native.dense_masked}[route]
        if self.stop > self.start:
            fn(hidden_2d, self.weight, mask, logits=local_logits, top_key=keys, vocab_offset=self.start)
        else:
            keys.fill_(KEY_SIGN)
        merge_top1_keys(keys, self.group)
        top_value = torch.empty(batch, device=dev, dtype=torch.float32)
        top_index = torch.empty(batch, device=dev, dtype=torch.int64)
        _native.top1_from_keys(keys, top_value, top_index)
        logits = gather_logits(local_logits, self.vocab, self.group) if full_logits else None
        return top_value, top_index, logits

    def sample(self, hidden: torch.Tensor, bitmask_gpu: torch.Tensor, *, seeds: torch.Tensor, step: int,
               temperature: float = 1.0):
        """Grammar-conditioned sampling over the whole vocabulary from the row
        shards: every rank runs the fused sampler on its shard (its Gumbel
        noise is keyed by global token ids), then one integer-MAX all-reduce
        of the per-request sample keys and greedy keys and an all-gather of
        the per-shard log-sum-exps (merged by gsp_merge_logsumexp). The token
        ids equal a single-GPU grammar_sample over the full head bit for bit;
        the log-sum-exp agrees to fp32 rounding. Returns a SampleResult
        (logits None)."""
        from .triton_runtime import SampleResult
        hidden_2d = hidden.reshape(1, -1) if hidden.ndim == 1 else hidden
        batch = hidden_2d.shape[0]
        dev = hidden.device
        mask = self.local_mask(bitmask_gpu.reshape(batch, -1))
        skey = torch.empty(batch, device=dev, dtype=torch.int64)
        tkey = torch.empty(batch, device=dev, dtype=torch.int64)
        lse = torch.empty(batch, device=dev, dtype=torch.float32)
        sidx = torch.empty(batch, device=dev, dtype=torch.int64)
        if self.stop > self.start:
            _native.row_sparse_sample(hidden_2d, self.weight, mask, seeds.contiguous(), step, temperature, sidx,
                                      sample_logsumexp=lse, vocab_offset=self.start, sample_key=skey, top_key=tkey)
        else:
            skey.fill_(KEY_SIGN)
            tkey.fill_(KEY_SIGN)
            lse.fill_(float("-inf"))
        merge_top1_keys(skey, self.group)
        merge_top1_keys(tkey, self.group)
        if dist.is_initialized() and dist.get_world_size(self.group) > 1:
            parts = [torch.empty_like(lse) for _ in range(dist.get_world_size(self.group))]
            dist.all_gather(parts, lse, group=self.group)
            stacked = torch.stack(parts)
        else:
            stacked = lse.reshape(1, batch)
        out_lse = torch.empty(batch, device=dev, dtype=torch.float32)
        _native.merge_logsumexp(stacked.contiguous(), out_lse)
        token_ids = torch.empty(batch, device=dev, dtype=torch.int64)
        _native.top1_from_keys(skey, None, token_ids)
        top_value = torch.empty(batch, device=dev, dtype=torch.float32)
        top_index = torch.empty(batch, device=dev, dtype=torch.int64)
        _native.top1_from_keys(tkey, top_value, top_index)
        return SampleResult(token_ids, out_lse, top_value, top_index, None)
