"""Drop-in replacement for the reference's ``gsp.triton_runtime`` module.

The module name, function names, signatures, return values, route strings and
ValueError messages follow gsp/triton_runtime.py of
StealthEyeLLC/grammar-sparse-projection, so a decode loop written against the
reference runs unchanged. The computation underneath is not Triton: every
projection is one of the hand-written sm_100a CUDA kernels of libgsp_b200.so,
reached through its C ABI (include/gsp_b200.h):

  bitmask_sparse_logits      -> gsp_row_sparse_logits   (warp-streamed legal rows)
  bitmask_block_gemm_logits  -> gsp_block_gemm_logits   (tcgen05 over active tiles)
  dense_masked_logits        -> gsp_dense_masked_logits (tcgen05 over all tiles)

The block-size keyword arguments of the reference are accepted for signature
compatibility and ignored: tiling is fixed by the B200 kernels.

Differences from the reference, all deliberate:
  * the bitmask row stride is the tensor's real stride, so a mask wider than
    ceil(V/32) words is read correctly for every request (the reference kernels
    assume a stride of ceil(V/32), gsp/triton_runtime.py:32,171);
  * dense_masked_logits validates its inputs like the other two entry points;
  * extra entry points below the reference API return the fused greedy top-1,
    compact legal logits and device-side density statistics.
"""
from __future__ import annotations

from typing import NamedTuple

import torch

from . import _native
from ._native import TILE_ROWS

__all__ = [
    "bitmask_sparse_logits",
    "allocate_pinned_bitmask",
    "copy_bitmask_to_gpu",
    "bitmask_block_gemm_logits",
    "dense_masked_logits",
    "full_word_fraction_cpu",
    "adaptive_grammar_logits",
    "grammar_logits_with_top1",
    "grammar_sample",
    "SampleResult",
    "bitmask_compact_logits",
    "mask_stats",
    "choose_route",
    "ROUTES",
    "HeadResult",
    "grammar_head",
    "GroupedResult",
    "grouped_grammar_logits",
]

ROUTES = ("row-sparse", "block-sparse", "dense-mask")


# ---------------------------------------------------------------------------
# validation shared by the entry points (messages as in the reference)
# ---------------------------------------------------------------------------
def _sparse_inputs(hidden: torch.Tensor, weight: torch.Tensor, bitmask_gpu: torch.Tensor):
    """gsp/triton_runtime.py:75-109."""
    if hidden.device.type != "cuda" or weight.device.type != "cuda":
        raise ValueError("hidden and weight must be CUDA tensors")
    if bitmask_gpu.device.type != "cuda" or bitmask_gpu.dtype != torch.int32:
        raise ValueError("bitmask_gpu must be CUDA int32")
    if hidden.dtype != weight.dtype:
        raise ValueError("hidden and weight dtypes must match")
    if hidden.ndim == 1:
        hidden_2d = hidden.reshape(1, -1)
        squeeze = True
    elif hidden.ndim == 2:
        hidden_2d = hidden
        squeeze = hidden.shape[0] == 1
    else:
        raise ValueError("hidden must have shape [D] or [B, D]")
    if weight.ndim != 2:
        raise ValueError("weight must have shape [V, D]")
    vocab, hidden_dim = weight.shape
    batch = hidden_2d.shape[0]
    if hidden_2d.shape[1] != hidden_dim:
        raise ValueError("hidden dimension mismatch")
    if not hidden_2d.is_contiguous() or not weight.is_contiguous():
        raise ValueError("hidden and weight must be contiguous")
    mask_words = (vocab + 31) // 32
    if bitmask_gpu.ndim == 1:
        mask_2d = bitmask_gpu.reshape(1, -1)
    elif bitmask_gpu.ndim == 2:
        mask_2d = bitmask_gpu
    else:
        raise ValueError("bitmask must have shape [words] or [B, words]")
    if mask_2d.shape[0] != batch or mask_2d.shape[1] < mask_words:
        raise ValueError("bitmask shape does not match hidden batch/vocabulary")
    if not mask_2d.is_contiguous():
        raise ValueError("bitmask must be contiguous")
    _native.dtype_code(hidden.dtype)
    return hidden_2d, mask_2d, squeeze, batch, vocab


def _half_only(dtype: torch.dtype, what: str) -> None:
    """The device route selector, lane grouping and the sampler take
    half-precision inputs; float32 heads have one route (row-sparse), which
    the reference API functions run for every route name."""
    if dtype == torch.float32:
        raise ValueError(f"{what} takes float16 or bfloat16; float32 runs the row-sparse kernel on every route")


def _block_inputs(hidden: torch.Tensor, weight: torch.Tensor, bitmask_gpu: torch.Tensor):
    """gsp/triton_runtime.py:222-239."""
    if hidden.ndim != 2 or hidden.shape[0] < 2:
        raise ValueError("block GEMM path expects hidden shape [B,D] with B >= 2")
    if hidden.device.type != "cuda" or weight.device.type != "cuda":
        raise ValueError("hidden and weight must be CUDA tensors")
    if bitmask_gpu.device.type != "cuda" or bitmask_gpu.dtype != torch.int32:
        raise ValueError("bitmask_gpu must be CUDA int32")
    if hidden.dtype != weight.dtype:
        raise ValueError("hidden and weight dtypes must match")
    if not hidden.is_contiguous() or not weight.is_contiguous() or not bitmask_gpu.is_contiguous():
        raise ValueError("inputs must be contiguous")
    batch, hidden_dim = hidden.shape
    vocab, weight_hidden = weight.shape
    if hidden_dim != weight_hidden:
        raise ValueError("hidden dimension mismatch")
    mask_words = (vocab + 31) // 32
    if bitmask_gpu.ndim != 2 or bitmask_gpu.shape[0] != batch or bitmask_gpu.shape[1] < mask_words:
        raise ValueError("bitmask shape mismatch")
    _native.dtype_code(hidden.dtype)
    return batch, vocab


# ---------------------------------------------------------------------------
# reference API
# ---------------------------------------------------------------------------
def bitmask_sparse_logits(
    hidden: torch.Tensor,
    weight: torch.Tensor,
    bitmask_gpu: torch.Tensor,
    *,
    block_m: int = 32,
    block_k: int = 256,
) -> torch.Tensor:
    """Exact grammar-constrained logits without invalid-row matmul work.

    One or more hidden states share the LM-head weight, with one bitmask row
    per request. Illegal rows of the weight are never read and come out -inf.
    Output dtype = hidden dtype; shape [V] when hidden is 1-D or B == 1
    (gsp/triton_runtime.py:61-125).
    """
    del block_m, block_k
    hidden_2d, mask_2d, squeeze, batch, vocab = _sparse_inputs(hidden, weight, bitmask_gpu)
    out = torch.empty((batch, vocab), device=weight.device, dtype=hidden.dtype)
    _native.row_sparse(hidden_2d, weight, mask_2d, logits=out)
    return out[0] if squeeze else out


def allocate_pinned_bitmask(batch_size: int, vocab_size: int) -> torch.Tensor:
    """Pinned [B, ceil(V/32)] int32 host mask filled with -1 (gsp/triton_runtime.py:128-130)."""
    shape = (batch_size, (vocab_size + 31) // 32)
    return torch.full(shape, -1, dtype=torch.int32, pin_memory=True)


def copy_bitmask_to_gpu(
    bitmask_cpu: torch.Tensor,
    bitmask_gpu: torch.Tensor | None = None,
) -> torch.Tensor:
    """Asynchronous host-to-device copy of a pinned mask (gsp/triton_runtime.py:133-144)."""
    if bitmask_cpu.device.type != "cpu" or bitmask_cpu.dtype != torch.int32:
        raise ValueError("bitmask_cpu must be CPU int32")
    if not bitmask_cpu.is_pinned():
        raise ValueError("bitmask_cpu must be pinned for asynchronous transfer")
    if bitmask_gpu is None:
        bitmask_gpu = torch.empty_like(bitmask_cpu, device="cuda")
    bitmask_gpu.copy_(bitmask_cpu, non_blocking=True)
    return bitmask_gpu


def bitmask_block_gemm_logits(
    hidden: torch.Tensor,
    weight: torch.Tensor,
    bitmask_gpu: torch.Tensor,
    *,
    block_m: int = 16,
    block_n: int = 32,
    block_k: int = 64,
) -> torch.Tensor:
    """Batched grammar-aware LM head: tensor-core GEMM over only the 128-row
    vocabulary tiles that hold a legal token of some request
    (gsp/triton_runtime.py:212-258)."""
    del block_m, block_n, block_k
    batch, vocab = _block_inputs(hidden, weight, bitmask_gpu)
    out = torch.empty((batch, vocab), device=hidden.device, dtype=hidden.dtype)
    _native.block_gemm(hidden, weight, bitmask_gpu, logits=out)
    return out


def dense_masked_logits(
    hidden: torch.Tensor,
    weight: torch.Tensor,
    bitmask_gpu: torch.Tensor,
) -> torch.Tensor:
    """Dense LM head with the grammar mask fused into the GEMM epilogue
    (the result of F.linear + xgrammar's apply_token_bitmask_inplace,
    gsp/triton_runtime.py:285-308)."""
    if hidden.ndim == 1:
        hidden_2d = hidden.reshape(1, -1)
        squeeze = True
    elif hidden.ndim == 2:
        hidden_2d = hidden
        squeeze = hidden.shape[0] == 1
    else:
        raise ValueError("hidden must have shape [D] or [B,D]")
    if hidden.device.type != "cuda" or weight.device.type != "cuda":
        raise ValueError("hidden and weight must be CUDA tensors")
    if hidden.dtype != weight.dtype:
        raise ValueError("hidden and weight dtypes must match")
    if weight.ndim != 2 or hidden_2d.shape[1] != weight.shape[1]:
        raise ValueError("hidden dimension mismatch")
    if not hidden_2d.is_contiguous() or not weight.is_contiguous():
        raise ValueError("hidden and weight must be contiguous")
    batch, vocab = hidden_2d.shape[0], weight.shape[0]
    mask_2d = bitmask_gpu.reshape(batch, -1)
    if bitmask_gpu.device.type != "cuda" or bitmask_gpu.dtype != torch.int32:
        raise ValueError("bitmask_gpu must be CUDA int32")
    if mask_2d.shape[1] < (vocab + 31) // 32:
        raise ValueError("bitmask shape does not match hidden batch/vocabulary")
    out = torch.empty((batch, vocab), device=hidden.device, dtype=hidden.dtype)
    _native.dense_masked(hidden_2d, weight, mask_2d, logits=out)
    return out[0] if squeeze else out


def full_word_fraction_cpu(bitmask_cpu: torch.Tensor) -> list[float]:
    """Per request, the fraction of mask words equal to -1 (all 32 tokens
    legal), read from the host copy of the mask (gsp/triton_runtime.py:310-321)."""
    if bitmask_cpu.device.type != "cpu" or bitmask_cpu.dtype != torch.int32:
        raise ValueError("bitmask_cpu must be CPU int32")
    mask_2d = bitmask_cpu.reshape(bitmask_cpu.shape[0], -1)
    counts = (mask_2d == -1).sum(dim=1)
    denom = mask_2d.shape[1]
    return [float(x) / denom for x in counts.tolist()]


def _reference_route(batch: int, full_word_fraction, dense_full_word_threshold: float) -> str:
    """Routing rule of gsp/triton_runtime.py:341-353."""
    if full_word_fraction is not None:
        if len(full_word_fraction) != batch:
            raise ValueError("full_word_fraction length must equal batch")
        mean_full = sum(full_word_fraction) / batch
        all_near_dense = min(full_word_fraction) >= dense_full_word_threshold
        large_mixed_dense = batch >= 32 and mean_full >= 0.25
        if batch > 1 and (all_near_dense or large_mixed_dense):
            return "dense-mask"
    if batch == 1:
        return "row-sparse"
    return "block-sparse"


# B200 cost model of the three routes, in microseconds (see choose_route).
# Fitted to CUDA-graph timings on B200 at V=248,320, H=2,048 fp16, batch 1-32
# with 0.5%-legal clustered masks (row-sparse 12 / 18 / 37 us at batch 2 / 8 /
# 32; block-sparse 24 us up to batch 8, 55 us at batch 32 with 17% of the
# tiles active; dense 170 us).
B200_COST = {
    "hbm_gbs": 6000.0,             # legal rows and logits streamed by the row-sparse kernels
    "row_sparse_fixed_us": 9.0,    # launch, mask scan / slice-count exchange, top-1 merge
    "block_floor_us": 24.0,        # tile builder + tcgen05 pipeline: the least a block call costs
    "block_fixed_us": 10.0,
    "block_gbs": 3800.0,           # effective rate over the active tiles
    "dense_fixed_us": 5.0,
    "dense_gbs": 6000.0,
    "group_split_fixed_us": 10.0,  # lane-group split: row gathers, second route launch, un-permute
}


def choose_route(batch: int, vocab: int, hidden_dim: int, elem_bytes: int,
                 legal_counts, active_tiles: int, cost: dict | None = None) -> str:
    """B200-calibrated route choice from exact device-side statistics.

    Row-sparse reads every request's legal rows (sum_b k_b rows) and writes the
    B x V logits; block-sparse reads the union of active 128-row tiles once for
    all requests, with a floor for its builder and tensor-core pipeline; dense
    reads all of W. Each is a fixed latency plus its bytes at the rate measured
    for that kernel. Batch 1 always takes row-sparse, as in the reference.
    """
    c = dict(B200_COST, **(cost or {}))
    if batch == 1:
        return "row-sparse"
    row_bytes = hidden_dim * elem_bytes
    out_bytes = batch * vocab * elem_bytes
    t_row = c["row_sparse_fixed_us"] + (sum(int(k) for k in legal_counts) * row_bytes + out_bytes) / (c["hbm_gbs"] * 1e3)
    t_block = max(c["block_floor_us"],
                  c["block_fixed_us"] + min(active_tiles * TILE_ROWS, vocab) * row_bytes / (c["block_gbs"] * 1e3))
    t_dense = c["dense_fixed_us"] + vocab * row_bytes / (c["dense_gbs"] * 1e3)
    best = min((t_row, "row-sparse"), (t_block, "block-sparse"), (t_dense, "dense-mask"))
    return best[1]


def mask_stats(bitmask_gpu: torch.Tensor, vocab: int) -> dict:
    """Device-side density statistics of a [B, words] CUDA mask: legal token
    count and full-word count per request, and the number of 128-row vocabulary
    tiles active in the batch. Reads the three results back to the host (one
    small device-to-host copy)."""
    if bitmask_gpu.device.type != "cuda" or bitmask_gpu.dtype != torch.int32:
        raise ValueError("bitmask_gpu must be CUDA int32")
    mask_2d = bitmask_gpu.reshape(1, -1) if bitmask_gpu.ndim == 1 else bitmask_gpu
    batch = mask_2d.shape[0]
    buf = torch.empty(2 * batch + 1, dtype=torch.int32, device=bitmask_gpu.device)
    _native.mask_stats(mask_2d, vocab, legal_counts=buf[:batch], full_words=buf[batch:2 * batch],
                       active_tiles=buf[2 * batch:])
    host = buf.cpu().tolist()
    return {"legal_counts": host[:batch], "full_words": host[batch:2 * batch],
            "active_tiles": host[2 * batch], "total_tiles": (vocab + TILE_ROWS - 1) // TILE_ROWS}


def adaptive_grammar_logits(
    hidden: torch.Tensor,
    weight: torch.Tensor,
    bitmask_gpu: torch.Tensor,
    *,
    full_word_fraction: list[float] | None = None,
    dense_full_word_threshold: float = 0.80,
    policy: str = "reference",
) -> tuple[torch.Tensor, str]:
    """Exact grammar-conditioned output projection with route selection.

    Returns (logits, route), route in {"dense-mask", "row-sparse", "block-sparse"}.
    policy="reference" (default) applies the reference's rule to
    full_word_fraction (gsp/triton_runtime.py:324-353), so routes match the
    reference for the same inputs. policy="b200" measures the mask on the
    device (exact legal counts and active tiles) and applies choose_route.
    policy="device" lets the library's route selector kernel do both on the
    device (gsp_adaptive_logits; the same cost model), reading back only the
    chosen route (under CUDA-graph capture use grammar_head instead, whose
    route stays on the device). policy="grouped" also considers splitting the
    batch into two lane groups on different routes (grouped_grammar_logits);
    a split reports its routes joined by "+", e.g. "row-sparse+block-sparse".
    """
    batch = 1 if hidden.ndim == 1 else hidden.shape[0]
    if policy in ("grouped", "device"):
        _half_only(hidden.dtype, f"policy={policy!r}")
    if policy == "grouped":
        if full_word_fraction is not None and len(full_word_fraction) != batch:
            raise ValueError("full_word_fraction length must equal batch")
        _, _, squeeze, _, _ = _sparse_inputs(hidden, weight, bitmask_gpu)
        res = grouped_grammar_logits(hidden, weight, bitmask_gpu)
        return (res.logits[0] if squeeze else res.logits), "+".join(res.plan["routes"])
    if policy == "device":
        if full_word_fraction is not None and len(full_word_fraction) != batch:
            raise ValueError("full_word_fraction length must equal batch")
        hidden_2d, mask_2d, squeeze, batch, vocab = _sparse_inputs(hidden, weight, bitmask_gpu)
        out = torch.empty((batch, vocab), device=hidden.device, dtype=hidden.dtype)
        code = _native.adaptive(hidden_2d, weight, mask_2d, logits=out)
        if code < 0:
            raise ValueError("policy='device' reads the route back; under CUDA-graph capture use grammar_head")
        return (out[0] if squeeze else out), ROUTES[code]
    if policy == "reference":
        route = _reference_route(batch, full_word_fraction, dense_full_word_threshold)
    elif policy == "b200":
        if full_word_fraction is not None and len(full_word_fraction) != batch:
            raise ValueError("full_word_fraction length must equal batch")
        if batch == 1:
            route = "row-sparse"
        else:
            stats = mask_stats(bitmask_gpu, weight.shape[0])
            route = choose_route(batch, weight.shape[0], weight.shape[1], weight.element_size(),
                                 stats["legal_counts"], stats["active_tiles"])
    else:
        raise ValueError(f"unknown policy {policy!r}")
    if route == "dense-mask":
        return dense_masked_logits(hidden, weight, bitmask_gpu), route
    if route == "row-sparse":
        return bitmask_sparse_logits(hidden, weight, bitmask_gpu), route
    return bitmask_block_gemm_logits(hidden, weight, bitmask_gpu), route


# ---------------------------------------------------------------------------
# extensions beyond the reference API
# ---------------------------------------------------------------------------
def grammar_logits_with_top1(
    hidden: torch.Tensor,
    weight: torch.Tensor,
    bitmask_gpu: torch.Tensor,
    *,
    route: str = "row-sparse",
    return_logits: bool = True,
):
    """Masked logits plus the fused greedy top-1 of each request, in one launch.

    Returns (logits or None, top_value float32 [B], top_index int64 [B]).
    top_index equals logits.argmax(-1) exactly (ties to the lowest id), which
    replaces the separate argmax pass of the reference decode loop
    (benchmarks/qwen35_adaptive_paired.py:94). Shapes are [B, ...] always.
    """
    if route == "row-sparse":
        hidden_2d, mask_2d, _, batch, vocab = _sparse_inputs(hidden, weight, bitmask_gpu)
        fn = _native.row_sparse
    elif route in ("block-sparse", "dense-mask"):
        hidden_2d = hidden.reshape(1, -1) if hidden.ndim == 1 else hidden
        mask_2d = bitmask_gpu.reshape(hidden_2d.shape[0], -1)
        if route == "block-sparse":
            batch, vocab = _block_inputs(hidden_2d, weight, mask_2d) if hidden_2d.shape[0] >= 2 else (1, weight.shape[0])
        else:
            batch, vocab = hidden_2d.shape[0], weight.shape[0]
        fn = _native.block_gemm if route == "block-sparse" else _native.dense_masked
    else:
        raise ValueError(f"unknown route {route!r}")
    dev = hidden.device
    logits = torch.empty((batch, vocab), device=dev, dtype=hidden.dtype) if return_logits else None
    top_value = torch.empty(batch, device=dev, dtype=torch.float32)
    top_index = torch.empty(batch, device=dev, dtype=torch.int64)
    fn(hidden_2d, weight, mask_2d, logits=logits, top_value=top_value, top_index=top_index)
    return logits, top_value, top_index


class HeadResult(NamedTuple):
    logits: torch.Tensor | None  # [B, V] masked logits (None when not asked for)
    top_value: torch.Tensor      # float32 [B]: greedy top-1 logit
    top_index: torch.Tensor      # int64 [B]: greedy top-1 token
    route: torch.Tensor          # int32 [1] on the device: index into ROUTES


def grammar_head(hidden: torch.Tensor, weight: torch.Tensor, bitmask_gpu: torch.Tensor, *,
                 return_logits: bool = True, cost: dict | None = None,
                 out: HeadResult | None = None) -> HeadResult:
    """The whole grammar-conditioned head with the route chosen on the device.

    A selector kernel counts the batch's legal tokens and active 128-row tiles
    and applies the B200 cost model (choose_route's, with `cost` overriding
    fields of B200_COST); the chosen route computes the masked logits and
    fused greedy top-1. Nothing waits on the host when the call is captured
    in a CUDA graph (torch.cuda.graph): the capture holds a conditional node
    whose branches are the three routes, and each replay runs the one the
    selector picks for that replay's mask. Eager calls read the 4-byte route
    back. `out` reuses output tensors (for graph capture: allocate them before
    capturing). Warm up once outside capture on the capturing stream.
    """
    hidden_2d, mask_2d, _, batch, vocab = _sparse_inputs(hidden, weight, bitmask_gpu)
    _half_only(hidden.dtype, "grammar_head")
    dev = hidden.device
    if out is None:
        out = HeadResult(
            torch.empty((batch, vocab), device=dev, dtype=hidden.dtype) if return_logits else None,
            torch.empty(batch, device=dev, dtype=torch.float32),
            torch.empty(batch, device=dev, dtype=torch.int64),
            torch.zeros(1, device=dev, dtype=torch.int32))
    _native.adaptive(hidden_2d, weight, mask_2d, logits=out.logits, top_value=out.top_value,
                     top_index=out.top_index, route_out=out.route, cost=cost)
    return out


class GroupedResult(NamedTuple):
    logits: torch.Tensor | None  # [B, V] in the caller's request order
    top_value: torch.Tensor      # float32 [B]
    top_index: torch.Tensor      # int64 [B]
    plan: dict                   # split, routes, order and the modelled times


_ROUTE_FNS = {0: "row_sparse", 1: "block_gemm", 2: "dense_masked"}


def grouped_grammar_logits(hidden: torch.Tensor, weight: torch.Tensor, bitmask_gpu: torch.Tensor, *,
                           return_logits: bool = True, cost: dict | None = None) -> GroupedResult:
    """Masked logits and greedy top-1 with the batch split into two lane
    groups when that is cheaper (the reference's proposed lane grouping by
    density class, paper/draft.md:264-270).

    One native call (gsp_grouped_logits): the device profiles every request,
    orders the requests by the fill of their active 128-row tiles (scattered
    lanes first) and costs every split "first k | rest", each group on its
    cheapest route, against the best single route; the 32-byte plan header is
    read back; a split gathers the hidden and mask rows into group order,
    runs the two routes and permutes logits and top-1 back. Results equal
    the chosen routes' own (bit for bit); at most 256 requests; not
    capturable in a CUDA graph (grammar_head is).
    """
    hidden_2d, mask_2d, _, batch, vocab = _sparse_inputs(hidden, weight, bitmask_gpu)
    _half_only(hidden.dtype, "grouped_grammar_logits")
    if batch > _native.GROUP_MAX_BATCH:
        raise ValueError(f"grouped_grammar_logits takes at most {_native.GROUP_MAX_BATCH} requests")
    dev = hidden.device
    logits = torch.empty((batch, vocab), device=dev, dtype=hidden.dtype) if return_logits else None
    top_value = torch.empty(batch, device=dev, dtype=torch.float32)
    top_index = torch.empty(batch, device=dev, dtype=torch.int64)
    hdr = _native.grouped(hidden_2d, weight, mask_2d, logits=logits, top_value=top_value, top_index=top_index,
                          cost=cost)
    k = hdr[0]
    info = {"split": k, "single_route": ROUTES[hdr[3]], "single_us": hdr[4] / 1e3,
            "split_us": hdr[5] / 1e3 if hdr[5] >= 0 else None,
            "routes": (ROUTES[hdr[1]], ROUTES[hdr[2]]) if k else (ROUTES[hdr[3]],)}
    return GroupedResult(logits, top_value, top_index, info)


class SampleResult(NamedTuple):
    token_ids: torch.Tensor   # int64 [B]: sampled token per request
    logsumexp: torch.Tensor   # float32 [B]: log sum exp(legal logits / T)
    top_value: torch.Tensor   # float32 [B]: greedy top-1 logit
    top_index: torch.Tensor   # int64 [B]: greedy top-1 token
    logits: torch.Tensor | None


def grammar_sample(hidden: torch.Tensor, weight: torch.Tensor, bitmask_gpu: torch.Tensor, *,
                   seeds: torch.Tensor, step: int, temperature: float = 1.0,
                   return_logits: bool = False, route: str = "row-sparse") -> SampleResult:
    """Grammar-conditioned fused sampler: one launch projects the legal rows
    and draws each request's next token from softmax(logits / temperature)
    over its legal tokens, without writing vocabulary-shaped logits unless
    asked (the "fused grammar-aware sampler" the reference's paper leaves
    open, paper/draft.md section 6.4).

    The draw is Gumbel-max over the dtype-rounded legal logits with Philox
    noise keyed by seeds[b] (CUDA int64 [B], read as uint64) and counted by
    (token id, step): the same (seeds, step) reproduce the same tokens, on any
    route decomposition; use a new step per decode step. logsumexp gives the
    sampled token's log-probability, logit / temperature - logsumexp. The
    greedy top-1 comes with it. Shapes are [B, ...] always. route picks the
    projection: "row-sparse" (legal rows only), "block-sparse" (tensor-core
    tiles holding a legal token) or "dense-mask" (every tile); each draws from
    the same contract, noise computed for legal tokens only.
    """
    if route not in ROUTES:
        raise ValueError(f"unknown route {route!r}")
    hidden_2d, mask_2d, _, batch, vocab = _sparse_inputs(hidden, weight, bitmask_gpu)
    _half_only(hidden.dtype, "grammar_sample")
    if seeds.device.type != "cuda" or seeds.dtype != torch.int64 or seeds.numel() != batch:
        raise ValueError("seeds must be a CUDA int64 tensor with one seed per request")
    if not (temperature > 0.0) or temperature == float("inf"):
        raise ValueError("temperature must be positive and finite")
    dev = hidden.device
    logits = torch.empty((batch, vocab), device=dev, dtype=hidden.dtype) if return_logits else None
    token_ids = torch.empty(batch, device=dev, dtype=torch.int64)
    lse = torch.empty(batch, device=dev, dtype=torch.float32)
    top_value = torch.empty(batch, device=dev, dtype=torch.float32)
    top_index = torch.empty(batch, device=dev, dtype=torch.int64)
    _native.row_sparse_sample(hidden_2d, weight, mask_2d, seeds.contiguous(), step, temperature, token_ids,
                              sample_logsumexp=lse, logits=logits, top_value=top_value, top_index=top_index,
                              route=route)
    return SampleResult(token_ids, lse, top_value, top_index, logits)


def bitmask_compact_logits(hidden: torch.Tensor, weight: torch.Tensor, bitmask_gpu: torch.Tensor,
                           *, capacity: int | None = None):
    """Compact legal logits straight from the bitmask: returns
    (token_ids int64 [N], logits [N], offsets int64 [B+1]); request b owns
    positions offsets[b]:offsets[b+1], token ids ascending. Without
    `capacity`, the legal count is measured on the device first (one sync)."""
    hidden_2d, mask_2d, _, batch, vocab = _sparse_inputs(hidden, weight, bitmask_gpu)
    dev = hidden.device
    if capacity is None:
        capacity = int(sum(mask_stats(mask_2d, vocab)["legal_counts"]))
    logits = torch.empty(max(capacity, 1), device=dev, dtype=hidden.dtype)
    ids = torch.empty(max(capacity, 1), device=dev, dtype=torch.int64)
    offsets = torch.empty(batch + 1, device=dev, dtype=torch.int64)
    _native.row_sparse_compact(hidden_2d, weight, mask_2d, logits[:capacity] if capacity else None,
                               ids, offsets)
    return ids[:capacity], logits[:capacity], offsets
