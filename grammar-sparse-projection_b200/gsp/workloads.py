"""Seeded synthetic workloads of the grammar-conditioned LM head and host-side
mask statistics (numpy only).

The reference measures on grammar traces from xgrammar and HF tokenizers; here
legal-token sets with the same densities and shapes are drawn from seeded
generators: uniform sets (tests/test_triton_block_gemm.py:16-22 of the
reference draws its block-GEMM masks this way) and sets packed into a few
contiguous runs (enum-like grammar states). Masks use the reference's packed
layout: int32 words, token v legal iff bit v % 32 of word v // 32 is set
(gsp/triton_runtime.py:33-35).

The benchmark draws its inputs from here; the test oracle loads this file for
the same generators, so tests and benchmark see the same distributions.
"""
from __future__ import annotations

import numpy as np


def mask_words(vocab: int) -> int:
    """Words per request row: ceil(V/32)."""
    return (vocab + 31) // 32


def pack_bitmask(legal: np.ndarray) -> np.ndarray:
    """bool [B, V] -> packed int32 [B, ceil(V/32)], LSB-first."""
    legal = np.asarray(legal, dtype=bool)
    if legal.ndim == 1:
        legal = legal.reshape(1, -1)
    b, v = legal.shape
    padded = np.zeros((b, mask_words(v) * 32), dtype=np.uint8)
    padded[:, :v] = legal
    return np.packbits(padded, axis=1, bitorder="little").view("<u4").view(np.int32).reshape(b, mask_words(v))


def unpack_bitmask(mask, vocab: int) -> np.ndarray:
    """Packed int32 mask [B, >= ceil(V/32)] -> bool [B, V]; words beyond
    ceil(V/32) and bits >= V are ignored."""
    m = np.asarray(mask)
    if m.ndim == 1:
        m = m.reshape(1, -1)
    m = np.ascontiguousarray(m[:, :mask_words(vocab)]).astype(np.int32, copy=False).view(np.uint32)
    bits = np.unpackbits(m.astype("<u4", copy=False).view(np.uint8).reshape(m.shape[0], -1), axis=1,
                         bitorder="little")
    return bits[:, :vocab].astype(bool)


def uniform_legal_ids(rng: np.random.Generator, vocab: int, k: int) -> np.ndarray:
    """k distinct token ids drawn uniformly, sorted."""
    return np.sort(rng.choice(vocab, size=k, replace=False))


def clustered_legal_ids(rng: np.random.Generator, vocab: int, k: int, max_runs: int) -> np.ndarray:
    """k distinct token ids packed into 1..max_runs contiguous runs at random
    non-overlapping positions."""
    k = int(min(max(k, 0), vocab))
    if k == 0:
        return np.zeros(0, dtype=np.int64)
    runs = int(rng.integers(1, max(1, min(max_runs, k)) + 1))
    cuts = (np.sort(rng.choice(np.arange(1, k), size=runs - 1, replace=False)) if runs > 1
            else np.zeros(0, dtype=np.int64))
    lengths = np.diff(np.concatenate([[0], cuts, [k]])).astype(np.int64)
    gaps = rng.multinomial(vocab - k, np.ones(runs + 1) / (runs + 1))
    ids, pos = [], 0
    for r in range(runs):
        pos += int(gaps[r])
        ids.append(np.arange(pos, pos + lengths[r], dtype=np.int64))
        pos += int(lengths[r])
    return np.concatenate(ids)


def make_batch_mask(rng: np.random.Generator, batch: int, vocab: int, k_per_request,
                    *, clustered: bool = False, max_runs: int = 64) -> np.ndarray:
    """Packed int32 mask [batch, ceil(V/32)] with the given legal counts."""
    ks = list(k_per_request) if np.ndim(k_per_request) else [int(k_per_request)] * batch
    legal = np.zeros((batch, vocab), dtype=bool)
    for b, k in enumerate(ks):
        ids = clustered_legal_ids(rng, vocab, k, max_runs) if clustered else uniform_legal_ids(rng, vocab, k)
        legal[b, ids] = True
    return pack_bitmask(legal)


def mixed_batch_mask(rng: np.random.Generator, batch: int, vocab: int, constrained_fraction: float, *,
                     dense_density: float = 0.95, sparse_density: float = 0.002, max_runs: int = 16) -> np.ndarray:
    """Mixed-density batch of the dispatcher sweep: round(fraction * batch)
    requests at random positions are constrained (sparse_density of the tokens
    legal, in <= max_runs clustered runs), the others near-unconstrained
    (dense_density legal, drawn uniformly)."""
    n_con = int(round(constrained_fraction * batch))
    legal = np.zeros((batch, vocab), dtype=bool)
    order = rng.permutation(batch)
    for j, b in enumerate(order):
        ids = (clustered_legal_ids(rng, vocab, int(sparse_density * vocab), max_runs) if j < n_con
               else uniform_legal_ids(rng, vocab, int(dense_density * vocab)))
        legal[b, ids] = True
    return pack_bitmask(legal)


def legal_counts(mask, vocab: int) -> np.ndarray:
    """Legal tokens per request."""
    return unpack_bitmask(mask, vocab).sum(axis=1)


def active_tiles(mask, vocab: int, tile_rows: int = 128) -> int:
    """Number of tile_rows-row vocabulary tiles with a legal token in any request."""
    legal = unpack_bitmask(np.asarray(mask).reshape(np.asarray(mask).shape[0], -1), vocab)
    ntiles = (vocab + tile_rows - 1) // tile_rows
    padded = np.zeros(ntiles * tile_rows, dtype=bool)
    padded[:vocab] = legal.any(axis=0)
    return int(padded.reshape(ntiles, tile_rows).any(axis=1).sum())
