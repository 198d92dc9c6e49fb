"""CPU oracle for the grammar-conditioned LM-head projection.

TEST INFRASTRUCTURE ONLY. Nothing in the product path imports this module:
only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline and
reference arms use it, and only as the checker or the timed CPU baseline.

It restates, in numpy (bit arithmetic) and float64 torch-CPU dot products, the
reference's algorithm for this path (StealthEyeLLC/grammar-sparse-projection):

  * bitmask convention          gsp/triton_runtime.py:33-35  (LSB-first, int32 words)
  * row-sparse logits           gsp/triton_runtime.py:15-58, 61-125
  * block-GEMM logits           gsp/triton_runtime.py:147-209, 212-258
  * dense + mask                gsp/triton_runtime.py:285-308 (F.linear then
                                xgrammar apply_token_bitmask_inplace)
  * full-word fraction          gsp/triton_runtime.py:310-321
  * adaptive route choice       gsp/triton_runtime.py:324-353
  * constrained_projection      gsp/runtime.py:16-51
  * greedy top-1                benchmarks/qwen35_adaptive_paired.py:94 (argmax,
                                first maximal index)

Parity is pinned by tests/golden/*.npz, produced by tests/golden/make_golden.py
from the reference's own code (its Triton kernels under the Triton CPU
interpreter, its gsp.runtime on CPU tensors, xgrammar's CPU mask kernel).
"""
from __future__ import annotations

import math
import os
from dataclasses import dataclass

import numpy as np
import torch

# Grading tolerances for fp16/bf16 logits with fp32 accumulation.
RTOL = 2e-3
ATOL = 2e-3


# ---------------------------------------------------------------------------
# bitmask helpers
# ---------------------------------------------------------------------------
def mask_words(vocab: int) -> int:
    """Words per request row: ceil(V/32) (gsp/triton_runtime.py:99)."""
    return (vocab + 31) // 32


def unpack_bitmask(mask, vocab: int) -> np.ndarray:
    """Packed int32 mask [B, >=ceil(V/32)] -> bool [B, V], LSB-first.

    Token v of request b is legal iff bit v%32 of word v//32 is set
    (gsp/triton_runtime.py:33-35; pinned by tests/test_triton_sparse.py:16-20
    of the reference). Words beyond ceil(V/32) and bits >= V are ignored.
    """
    m = np.asarray(mask)
    if m.ndim == 1:
        m = m.reshape(1, -1)
    words = mask_words(vocab)
    m = np.ascontiguousarray(m[:, :words]).astype(np.int32, copy=False).view(np.uint32)
    as_bytes = m.astype("<u4", copy=False).view(np.uint8).reshape(m.shape[0], -1)
    bits = np.unpackbits(as_bytes, axis=1, bitorder="little")
    return bits[:, :vocab].astype(bool)


def pack_bitmask(legal: np.ndarray) -> np.ndarray:
    """bool [B, V] -> packed int32 [B, ceil(V/32)] (inverse of unpack_bitmask)."""
    legal = np.asarray(legal, dtype=bool)
    if legal.ndim == 1:
        legal = legal.reshape(1, -1)
    b, v = legal.shape
    words = mask_words(v)
    padded = np.zeros((b, words * 32), dtype=np.uint8)
    padded[:, :v] = legal
    packed = np.packbits(padded, axis=1, bitorder="little")
    return packed.view("<u4").view(np.int32).reshape(b, words)


def ids_to_bitmask(ids, vocab: int, batch: int = 1) -> np.ndarray:
    """Token ids -> packed mask (the builder of tests/test_triton_sparse.py:16-20)."""
    legal = np.zeros((batch, vocab), dtype=bool)
    legal[:, np.asarray(ids, dtype=np.int64)] = True
    return pack_bitmask(legal)


# ---------------------------------------------------------------------------
# projection
# ---------------------------------------------------------------------------
def _as_cpu(t) -> torch.Tensor:
    if isinstance(t, np.ndarray):
        return torch.from_numpy(t)
    return t.detach().to("cpu")


def masked_logits_exact(hidden, weight, mask) -> torch.Tensor:
    """Exact masked logits in float64 (no rounding): dot products of the
    low-precision inputs, -inf where illegal; mask=None means all legal.
    Shape [B, V], or [V] for 1-D hidden.

    The reference's three routes (gsp/triton_runtime.py:15-58, 147-209,
    285-308) all accumulate in fp32 and round once to the input dtype, so a
    correct kernel output lies within half an output ulp (plus fp32
    accumulation error) of these values.
    """
    h = _as_cpu(hidden)
    w = _as_cpu(weight)
    squeeze = h.ndim == 1
    h2 = h.reshape(1, -1) if squeeze else h
    batch, vocab = h2.shape[0], w.shape[0]
    if mask is None:
        legal = np.ones((batch, vocab), dtype=bool)
    else:
        m = mask.detach().cpu().numpy() if isinstance(mask, torch.Tensor) else np.asarray(mask)
        legal = unpack_bitmask(m.reshape(batch, -1), vocab)
    out = torch.full((batch, vocab), float("-inf"), dtype=torch.float64)
    h64 = h2.to(torch.float64)
    chunk = 16384
    for b in range(batch):
        ids = torch.from_numpy(np.flatnonzero(legal[b]))
        for s in range(0, ids.numel(), chunk):
            sel = ids[s:s + chunk]
            out[b, sel] = w[sel].to(torch.float64) @ h64[b]
    return out[0] if squeeze else out


def masked_logits(hidden, weight, mask, *, out_dtype=None) -> torch.Tensor:
    """masked_logits_exact rounded once (round-to-nearest-even) to the output
    dtype (the input dtype by default): the materialised logits of the
    reference's routes."""
    exact = masked_logits_exact(hidden, weight, mask)
    return exact.to(out_dtype or _as_cpu(hidden).dtype)


def ulp(dtype: torch.dtype, x) -> torch.Tensor:
    """Spacing of `dtype` values at magnitude |x| (normal range)."""
    mant = {torch.float16: 10, torch.bfloat16: 7, torch.float32: 23}[dtype]
    ax = torch.as_tensor(x, dtype=torch.float64).abs().clamp_min(2.0 ** -14)
    return torch.exp2(torch.floor(torch.log2(ax)) - mant)


def top1(logits) -> tuple[torch.Tensor, torch.Tensor]:
    """Greedy top-1 per row: (value, index), first maximal index (torch.argmax)."""
    lg = _as_cpu(logits)
    if lg.ndim == 1:
        lg = lg.reshape(1, -1)
    idx = lg.float().argmax(-1)
    return lg.float().gather(1, idx[:, None])[:, 0], idx


def value_bound(ref, dtype: torch.dtype | None, *, rtol: float = RTOL, atol: float = ATOL) -> torch.Tensor:
    """Allowed |got - ref| for logits rounded to `dtype`:
    atol + max(rtol * |ref|, ulp(ref) / 2).

    For fp16 the half-ulp term never exceeds rtol * |ref| (unit roundoff
    2^-11), so this is exactly the stated rtol/atol 2e-3 bound. bf16's unit
    roundoff is 2^-8 = 3.9e-3, coarser than rtol 2e-3: a correctly rounded
    bf16 logit may sit half an ulp from the exact value, which the bound admits.
    dtype=None applies the plain rtol/atol bound.
    """
    r = torch.as_tensor(ref, dtype=torch.float64).abs()
    rel = rtol * r
    if dtype in (torch.float16, torch.bfloat16):
        rel = torch.maximum(rel, 0.5 * ulp(dtype, r))
    return atol + rel


def top1_agrees(ref_logits, got_index, *, dtype: torch.dtype | None = None,
                rtol: float = RTOL, atol: float = ATOL) -> bool:
    """True iff each got index is the reference's argmax, or a legal token whose
    reference logit lies within the near-tie window of the reference maximum:
    atol + max(rtol * |max|, one output ulp) (two exact values up to one ulp
    apart can round to the same output value, and then the lowest id wins)."""
    ref = _as_cpu(ref_logits).double()
    if ref.ndim == 1:
        ref = ref.reshape(1, -1)
    got = _as_cpu(torch.as_tensor(got_index)).reshape(-1).long()
    for b in range(ref.shape[0]):
        r = ref[b]
        i_ref = int(r.argmax())
        i_got = int(got[b])
        if i_got == i_ref:
            continue
        best = float(r[i_ref])
        if not math.isfinite(best):
            return False
        val = float(r[i_got])
        window = atol + rtol * abs(best)
        if dtype in (torch.float16, torch.bfloat16):
            window = max(window, atol + float(ulp(dtype, best)))
        if not math.isfinite(val) or best - val > window:
            return False
    return True


def compare_logits(ref, got, *, dtype: torch.dtype | None = None, rtol: float = RTOL,
                   atol: float = ATOL) -> dict:
    """Parity report: legal support (the finite entries) must match exactly and
    every legal value must satisfy |got - ref| <= value_bound(ref, dtype).
    `ref` is normally masked_logits_exact (float64, unrounded)."""
    r = _as_cpu(ref).double()
    g = _as_cpu(got).double()
    support = bool(torch.equal(torch.isfinite(r), torch.isfinite(g)))
    neg_inf_ok = bool(torch.all(torch.isneginf(g) | torch.isfinite(g)))
    fin = torch.isfinite(r) & torch.isfinite(g)
    if fin.any():
        diff = (r[fin] - g[fin]).abs()
        max_abs = float(diff.max())
        ok_vals = bool(torch.all(diff <= value_bound(r[fin], dtype, rtol=rtol, atol=atol)))
    else:
        max_abs, ok_vals = 0.0, True
    return {"support": support and neg_inf_ok, "values": ok_vals, "max_abs": max_abs}


# ---------------------------------------------------------------------------
# host-side signals and routing
# ---------------------------------------------------------------------------
def full_word_fraction(mask) -> list[float]:
    """Fraction of words equal to -1 per request row (gsp/triton_runtime.py:310-321);
    the denominator is the stored row width."""
    m = np.asarray(mask)
    m = m.reshape(m.shape[0], -1)
    counts = (m.astype(np.int32) == -1).sum(axis=1)
    return [float(x) / m.shape[1] for x in counts.tolist()]


def adaptive_route(batch: int, full_word_fraction_values=None,
                   dense_full_word_threshold: float = 0.80) -> str:
    """Route name chosen by gsp/triton_runtime.py:341-353."""
    if full_word_fraction_values is not None:
        if len(full_word_fraction_values) != batch:
            raise ValueError("full_word_fraction length must equal batch")
        mean_full = sum(full_word_fraction_values) / batch
        all_near_dense = min(full_word_fraction_values) >= dense_full_word_threshold
        large_mixed_dense = batch >= 32 and mean_full >= 0.25
        if batch > 1 and (all_near_dense or large_mixed_dense):
            return "dense-mask"
    if batch == 1:
        return "row-sparse"
    return "block-sparse"


def active_tiles(mask, vocab: int, tile_rows: int = 128) -> int:
    """Number of tile_rows-row vocabulary tiles with a legal token in any request."""
    legal = unpack_bitmask(np.asarray(mask).reshape(np.asarray(mask).shape[0], -1), vocab)
    any_legal = legal.any(axis=0)
    ntiles = (vocab + tile_rows - 1) // tile_rows
    padded = np.zeros(ntiles * tile_rows, dtype=bool)
    padded[:vocab] = any_legal
    return int(padded.reshape(ntiles, tile_rows).any(axis=1).sum())


@dataclass(frozen=True)
class OracleProjection:
    token_ids: torch.Tensor
    logits: torch.Tensor
    mode: str


def constrained_projection(hidden, weight, allowed_ids, *, dense_threshold: float = 0.30) -> OracleProjection:
    """gsp/runtime.py:16-51 restated on CPU (float64 dots, rounded to the input dtype)."""
    w = _as_cpu(weight)
    h = _as_cpu(hidden)
    vocab = w.shape[0]
    if allowed_ids is None:
        ids = torch.arange(vocab, dtype=torch.long)
        return OracleProjection(ids, masked_logits(h, w, None), "dense-unconstrained")
    ids = _as_cpu(torch.as_tensor(allowed_ids)).to(torch.long)
    if ids.ndim != 1:
        raise ValueError("allowed_ids must be one-dimensional")
    if ids.numel() == 0:
        raise ValueError("grammar produced an empty legal-token set")
    if torch.any(ids < 0) or torch.any(ids >= vocab):
        raise ValueError("allowed_ids contains an out-of-range token ID")
    ids = torch.unique(ids, sorted=True)
    density = ids.numel() / vocab
    mode = "dense-selected" if density >= dense_threshold else "sparse-gather"
    rows = w[ids].to(torch.float64)
    h2 = h.reshape(1, -1) if h.ndim == 1 else h
    logits = (h2.to(torch.float64) @ rows.T).to(h.dtype)
    if h.ndim == 1:
        logits = logits[0]
    return OracleProjection(ids, logits, mode)


# ---------------------------------------------------------------------------
# seeded synthetic inputs (the workload generators shared by tests and bench)
# ---------------------------------------------------------------------------
# Seeded legal-set generators: the package's workload module (numpy only),
# loaded from its file so that this module never imports a package named
# `gsp` (the golden-vector script imports the reference's).
def _load_workloads():
    import importlib.util
    path = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                        "grammar-sparse-projection_b200", "gsp", "workloads.py")
    spec = importlib.util.spec_from_file_location("gsp_b200_workloads", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


_workloads = _load_workloads()
uniform_legal_ids = _workloads.uniform_legal_ids
clustered_legal_ids = _workloads.clustered_legal_ids
make_batch_mask = _workloads.make_batch_mask


# ---------------------------------------------------------------------------
# fused sampler (no counterpart in the reference; its paper names it as the
# next step, paper/draft.md section 6.4). Restates the contract the kernels
# implement, independently, for the checker:
#   u = ((Philox4x32-10({v, offset lo, offset hi, 0}, {seed lo, seed hi}).word0 >> 8) + 0.5) / 2^24
#   g = -log(-log(u)); s = x * (1/T) + g (fp32); sample = argmax s (lowest id on ties)
#   lse = log sum exp(x / T)
# ---------------------------------------------------------------------------
_PHILOX_M0, _PHILOX_M1 = 0xD2511F53, 0xCD9E8D57  # Salmon et al., SC 2011
_PHILOX_W0, _PHILOX_W1 = 0x9E3779B9, 0xBB67AE85
_U32 = np.uint64(0xFFFFFFFF)


def philox4x32_10(counters, key0: int, key1: int) -> np.ndarray:
    """Philox4x32-10 of each row of counters [N, 4] (uint32) under key
    (key0, key1): ten rounds, key bumped by the Weyl constants between them."""
    c = np.asarray(counters, dtype=np.uint64).reshape(-1, 4)
    c0, c1, c2, c3 = c[:, 0].copy(), c[:, 1].copy(), c[:, 2].copy(), c[:, 3].copy()
    k0, k1 = np.uint64(key0 & 0xFFFFFFFF), np.uint64(key1 & 0xFFFFFFFF)
    for _ in range(10):
        p0 = c0 * np.uint64(_PHILOX_M0)
        p1 = c2 * np.uint64(_PHILOX_M1)
        c0, c1, c2, c3 = (p1 >> np.uint64(32)) ^ c1 ^ k0, p1 & _U32, (p0 >> np.uint64(32)) ^ c3 ^ k1, p0 & _U32
        k0 = (k0 + np.uint64(_PHILOX_W0)) & _U32
        k1 = (k1 + np.uint64(_PHILOX_W1)) & _U32
    return np.stack([c0, c1, c2, c3], axis=1).astype(np.uint32)


def gumbel_noise(seed: int, offset: int, ids) -> np.ndarray:
    """fp32 Gumbel noise of global token ids for one request's seed and step."""
    ids = np.asarray(ids, dtype=np.uint64)
    ctr = np.stack([ids & _U32, np.full_like(ids, offset & 0xFFFFFFFF), np.full_like(ids, (offset >> 32) & 0xFFFFFFFF),
                    np.zeros_like(ids)], axis=1)
    word0 = philox4x32_10(ctr, seed & 0xFFFFFFFF, (seed >> 32) & 0xFFFFFFFF)[:, 0]
    u = ((word0 >> np.uint32(8)).astype(np.float32) + np.float32(0.5)) * np.float32(2.0 ** -24)
    return (-np.log(-np.log(u))).astype(np.float32)


def sample_reference(hidden, weight, mask, dtype: torch.dtype, temperature: float, seeds, offset: int,
                     vocab_offset: int = 0):
    """Per request: (sampled id or 0, logsumexp in float64, perturbed scores
    of the legal tokens as float32, the legal ids). x is the exact logit
    rounded to `dtype` (what the materialised logits hold)."""
    exact = masked_logits_exact(hidden, weight, mask)
    rounded = exact.to(dtype).float().numpy()
    inv_t = np.float32(1.0) / np.float32(temperature)
    out = []
    for b in range(rounded.shape[0]):
        legal = np.flatnonzero(np.isfinite(rounded[b]))
        if legal.size == 0:
            out.append((0, float("-inf"), np.zeros(0, np.float32), legal))
            continue
        y = rounded[b, legal].astype(np.float32) * inv_t
        scores = y + gumbel_noise(int(seeds[b]), offset, legal + vocab_offset)
        pick = int(legal[int(np.argmax(scores))]) + vocab_offset
        y64 = y.astype(np.float64)
        lse = float(y64.max() + np.log(np.exp(y64 - y64.max()).sum()))
        out.append((pick, lse, scores, legal + vocab_offset))
    return out


def cpu_row_sparse_step(hidden: np.ndarray, weight: np.ndarray, mask: np.ndarray, vocab: int) -> tuple[np.ndarray, np.ndarray]:
    """One CPU step of the reference's row-sparse semantics for the timed CPU
    baseline: decode the bitmask, gather legal rows (gsp/runtime.py:50-51),
    fp32 dot products, -inf fill and greedy top-1. Returns (logits fp32, top1 idx)."""
    legal = unpack_bitmask(mask, vocab)
    h = np.asarray(hidden, dtype=np.float32).reshape(legal.shape[0], -1)
    out = np.full(legal.shape, -np.inf, dtype=np.float32)
    for b in range(legal.shape[0]):
        ids = np.flatnonzero(legal[b])
        if ids.size:
            out[b, ids] = weight[ids].astype(np.float32) @ h[b]
    return out, out.argmax(axis=1)


def config0_inputs(seed: int = 0, vocab: int = 32768, hidden: int = 1024, density: float = 0.01):
    """CPU plumbing configuration: fp32 W ~ N(0, 0.02) [V, H], h ~ N(0, 1) [1, H],
    int(density * V) legal ids drawn uniformly; numpy default_rng(seed)."""
    rng = np.random.default_rng(seed)
    w = torch.from_numpy(rng.standard_normal((vocab, hidden), dtype=np.float32) * np.float32(0.02))
    h = torch.from_numpy(rng.standard_normal((1, hidden), dtype=np.float32))
    ids = uniform_legal_ids(rng, vocab, int(vocab * density))
    return w, h, ids


# ---------------------------------------------------------------------------
# golden-case input generators (shared by tests/golden/make_golden.py and tests)
# ---------------------------------------------------------------------------
TORCH_DTYPES = {"float16": torch.float16, "bfloat16": torch.bfloat16, "float32": torch.float32}


def recipe_mask(recipe: str, rng: np.random.Generator, batch: int, vocab: int, extra_words: int = 0) -> np.ndarray:
    """Packed mask [batch, ceil(V/32) + extra_words] from a '+'-separated recipe,
    cycled over the batch: zero | full (all words -1, tail bits set) | random
    (raw random words) | u<k> (k uniform ids) | c<k> (k ids in <= 16 runs) |
    first (only token 0, tests/test_adaptive_dispatch.py:30 of the reference)."""
    words = mask_words(vocab) + extra_words
    kinds = recipe.split("+")
    out = np.zeros((batch, words), dtype=np.int32)
    for b in range(batch):
        kind = kinds[b % len(kinds)]
        row = np.zeros(words, dtype=np.int32)
        if kind == "zero":
            pass
        elif kind == "full":
            row[:] = -1
        elif kind == "random":
            row[:] = rng.integers(-2**31, 2**31 - 1, size=words, dtype=np.int64).astype(np.int32)
        elif kind[0] in "uc":
            k = int(kind[1:])
            ids = uniform_legal_ids(rng, vocab, k) if kind[0] == "u" else clustered_legal_ids(rng, vocab, k, 16)
            legal = np.zeros(vocab, dtype=bool)
            legal[ids] = True
            row[: mask_words(vocab)] = pack_bitmask(legal)[0]
        elif kind == "first":
            row[0] = 1
        else:
            raise ValueError(kind)
        out[b] = row
    return out


def kernel_case_inputs(vocab: int, hidden: int, batch: int, dtype: str, seed: int, recipe: str,
                       extra_words: int = 0):
    """(weight [V,H], hidden [B,H], mask) for one golden kernel case; W, h ~ N(0,1)
    as in the reference's tests (tests/test_triton_sparse.py:29-30)."""
    rng = np.random.default_rng(seed)
    tdt = TORCH_DTYPES[dtype]
    w = torch.from_numpy(rng.standard_normal((vocab, hidden), dtype=np.float32)).to(tdt)
    h = torch.from_numpy(rng.standard_normal((batch, hidden), dtype=np.float32)).to(tdt)
    return w, h, recipe_mask(recipe, rng, batch, vocab, extra_words)


def projection_case_inputs(dtype: str, seed: int, vocab: int = 3000, hidden: int = 128, batch: int = 2):
    """(weight, hidden) for the small constrained_projection golden cases."""
    rng = np.random.default_rng(seed)
    tdt = TORCH_DTYPES[dtype]
    w = torch.from_numpy(rng.standard_normal((vocab, hidden), dtype=np.float32)).to(tdt)
    h = torch.from_numpy(rng.standard_normal((batch, hidden), dtype=np.float32)).to(tdt)
    return w, h


def tensor_sha256(t) -> str:
    """sha256 of a tensor's / array's raw bytes (used to detect generator drift)."""
    import hashlib
    if isinstance(t, torch.Tensor):
        t = t.detach().cpu().contiguous()
        a = t.view(torch.int16).numpy() if t.dtype in (torch.float16, torch.bfloat16) else t.numpy()
    else:
        a = np.asarray(t)
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def bits16_to_tensor(bits: np.ndarray, dtype: str) -> torch.Tensor:
    """uint16 bit patterns -> fp16/bf16 tensor."""
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(TORCH_DTYPES[dtype])
