"""Host-side logic of the vocabulary-parallel head on CPU ranks (gloo, world 2):
shard bounds, top-1 key packing, the integer-MAX merge and the logit
all-gather, checked against the single-process oracle."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from gsp import vocab_parallel as vp
from oracle import gsp_oracle as O


def test_shard_bounds_cover_vocab():
    for vocab in (1, 31, 32, 1000, 248320, 262144, 151936):
        for world in (1, 2, 3, 4, 8):
            bounds = [vp.shard_bounds(vocab, world, r) for r in range(world)]
            assert bounds[0][0] == 0 and bounds[-1][1] == vocab
            for (a, b), (c, d) in zip(bounds, bounds[1:]):
                assert b == c and a % 32 == 0 and c % 32 == 0
            sizes = [b - a for a, b in bounds]
            assert max(sizes) - min(sizes) <= 32 or vocab % 32
    assert vp.shard_bounds(248320, 8, 3) == (93120, 124160)


def test_key_roundtrip_and_order():
    vals = torch.tensor([1.5, -2.0, 0.0, -0.0, float("-inf"), 3.25, 3.25], dtype=torch.float16).float()
    idx = torch.tensor([7, 3, 9, 2, 11, 40, 5])
    keys = vp.encode_keys(vals, idx)
    v, i = vp.decode_keys(keys)
    assert torch.equal(i, torch.where(vals == 0, idx, idx)) and torch.equal(v[vals != 0], vals[vals != 0])
    # larger value wins; equal values -> lower index wins; +0 == -0
    assert keys[6] > keys[5]
    assert keys[3] > keys[2]
    assert keys[4] > vp.encode_keys(torch.tensor([0.0]), torch.tensor([0]), torch.tensor([False]))[0]
    empty = vp.encode_keys(torch.zeros(1), torch.zeros(1, dtype=torch.long), torch.tensor([False]))
    ev, ei = vp.decode_keys(empty)
    assert ev.item() == float("-inf") and ei.item() == 0


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, case, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        vocab, hidden, batch, seed = case
        rng = np.random.default_rng(seed)
        w = torch.from_numpy(rng.standard_normal((vocab, hidden), dtype=np.float32)).half()
        h = torch.from_numpy(rng.standard_normal((batch, hidden), dtype=np.float32)).half()
        mask = O.make_batch_mask(rng, batch, vocab, [0, 1, 37, vocab // 3][:batch], clustered=True, max_runs=4)
        # a tie across the shard boundary: request 0 gets two identical rows
        lo, hi = vp.shard_bounds(vocab, world, rank)
        full = O.masked_logits(h, w, mask)
        local = full[:, lo:hi]
        fin = torch.isfinite(local)
        vals = torch.where(fin, local.float(), torch.full_like(local.float(), float("-inf")))
        loc_idx = vals.argmax(1)
        loc_val = vals.gather(1, loc_idx[:, None])[:, 0]
        keys = vp.encode_keys(loc_val, loc_idx + lo, fin.any(1))
        vp.merge_top1_keys(keys)
        gv, gi = vp.decode_keys(keys)
        ref_v, ref_i = O.top1(full)
        gathered = vp.gather_logits(local, vocab)
        q.put((rank, bool(torch.equal(gi, ref_i)), bool(torch.equal(gv, ref_v)),
               bool(torch.equal(gathered, full))))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("case", [(1000, 64, 4, 5), (4096, 32, 3, 6)])
def test_vocab_parallel_merge_gloo(case):
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, case, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, idx_ok, val_ok, gather_ok in results:
        assert idx_ok and val_ok and gather_ok, (rank, idx_ok, val_ok, gather_ok)


def test_tie_across_shards_prefers_lowest_global_index():
    keys_r0 = vp.encode_keys(torch.tensor([2.5]), torch.tensor([100]))
    keys_r1 = vp.encode_keys(torch.tensor([2.5]), torch.tensor([900]))
    merged = torch.maximum(keys_r0, keys_r1)
    _, idx = vp.decode_keys(merged)
    assert idx.item() == 100


def _sample_worker(rank, world, port, case, q):
    """One CPU rank of a sharded sampling step: the oracle's Gumbel-max keys of
    this rank's row shard (noise keyed by global token ids, as the sampler
    kernel keys it), merged across ranks by the integer-MAX all-reduce that
    VocabParallelHead.sample uses, and the shard log-sum-exps all-gathered and
    combined; both against the oracle's whole-vocabulary draw."""
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        vocab, hidden, batch, seed, temperature, step = case
        rng = np.random.default_rng(seed)
        w = torch.from_numpy(rng.standard_normal((vocab, hidden), dtype=np.float32) * 0.3).half()
        h = torch.from_numpy(rng.standard_normal((batch, hidden), dtype=np.float32)).half()
        ks = [0] + [int(k) for k in rng.integers(1, vocab // 10, size=batch - 1)]
        mask = O.make_batch_mask(rng, batch, vocab, ks, clustered=True, max_runs=6)
        seeds = [int(s) for s in rng.integers(1, 2 ** 62, size=batch)]
        lo, hi = vp.shard_bounds(vocab, world, rank)
        shard = O.sample_reference(h, w[lo:hi], np.ascontiguousarray(mask[:, lo // 32:(hi + 31) // 32]),
                                   torch.float16, temperature, seeds, step, vocab_offset=lo)
        vals = torch.tensor([float(s.max()) if ids.size else 0.0 for _, _, s, ids in shard], dtype=torch.float32)
        idx = torch.tensor([int(ids[int(np.argmax(s))]) if ids.size else 0 for _, _, s, ids in shard])
        valid = torch.tensor([ids.size > 0 for _, _, _, ids in shard])
        keys = vp.encode_keys(vals, idx, valid)
        vp.merge_top1_keys(keys)
        _, pick = vp.decode_keys(keys)
        lse = torch.tensor([lse for _, lse, _, _ in shard], dtype=torch.float64)
        parts = [torch.empty_like(lse) for _ in range(world)]
        dist.all_gather(parts, lse)
        stacked = torch.stack(parts)
        merged = torch.logsumexp(stacked, dim=0)
        full = O.sample_reference(h, w, mask, torch.float16, temperature, seeds, step)
        want_pick = torch.tensor([p for p, _, _, _ in full])
        want_lse = torch.tensor([l for _, l, _, _ in full], dtype=torch.float64)
        fin = torch.isfinite(want_lse)
        q.put((rank, bool(torch.equal(pick, want_pick)),
               bool(torch.equal(torch.isfinite(merged), fin)
                    and torch.allclose(merged[fin], want_lse[fin], rtol=1e-12, atol=1e-9))))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("case", [(3000, 32, 5, 21, 0.8, 3), (4099, 16, 4, 22, 1.3, 12345)])
def test_sampling_merge_gloo(case):
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_sample_worker, args=(r, world, port, case, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, pick_ok, lse_ok in results:
        assert pick_ok and lse_ok, (rank, pick_ok, lse_ok)


def test_check_exchange_raises_on_the_time_out_marker():
    """An in-kernel exchange whose wait ran out reports top_index -1 for every
    request; check_exchange turns that into ExchangeTimeout and passes real
    token ids (0 included: the id of an all -inf row) through."""
    from gsp import vocab_parallel as vp
    vp.check_exchange(torch.tensor([0, 5, 123456], dtype=torch.int64))
    with pytest.raises(vp.ExchangeTimeout):
        vp.check_exchange(torch.tensor([-1, -1], dtype=torch.int64))
