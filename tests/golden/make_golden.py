"""Generate the golden fixtures that pin the CPU oracle to the reference.

Runs ONLY where a reference checkout is available; its path is the one
required argument. The fixtures it writes are committed next to this script
and are all the tests need afterwards.

What is recorded, all produced by the reference's own code on this machine:
  * row_sparse_ref.npz   -- gsp/triton_runtime.py:15-58 (_bitmask_sparse_lm_head_kernel)
                            launched exactly as bitmask_sparse_logits does (:111-124),
                            under the Triton CPU interpreter (TRITON_INTERPRET=1)
  * block_gemm_ref.npz   -- gsp/triton_runtime.py:147-209 (_bitmask_block_gemm_kernel)
                            launched as bitmask_block_gemm_logits does (:241-257)
  * dense_mask_ref.npz   -- gsp/triton_runtime.py:302-307 (F.linear followed by
                            xgrammar.apply_token_bitmask_inplace; backend "cpu"
                            because this machine has no GPU)
  * projection_ref.npz   -- gsp/runtime.py:16-51 (constrained_projection) on CPU
                            tensors, incl. the 32,768 x 1,024 fp32 1% case
  * routes_ref.json      -- gsp/triton_runtime.py:324-353 route names with the
                            three route functions replaced by recorders, and
                            gsp/triton_runtime.py:310-321 full_word_fraction_cpu

Usage:  python tests/golden/make_golden.py /path/to/reference/checkout
"""
from __future__ import annotations

import json
import os
import sys

os.environ["TRITON_INTERPRET"] = "1"  # must precede the first triton import

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
if len(sys.argv) != 2 or not os.path.isdir(os.path.join(sys.argv[1], "gsp")):
    raise SystemExit("usage: python tests/golden/make_golden.py /path/to/reference/checkout")
REF = os.path.abspath(sys.argv[1])
sys.path.insert(0, REPO)
sys.path.insert(0, REF)

from oracle import gsp_oracle as O  # noqa: E402  (input generators only)

import gsp.runtime as ref_runtime  # noqa: E402  (the reference package)
import gsp.triton_runtime as ref_tr  # noqa: E402
import xgrammar as xgr  # noqa: E402

assert os.path.abspath(ref_tr.__file__).startswith(os.path.abspath(REF)), ref_tr.__file__

def bits16(t: torch.Tensor) -> np.ndarray:
    """fp16/bf16 tensor -> its raw uint16 bit pattern (numpy has no bf16)."""
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


# ---------------------------------------------------------------------------
# kernel cases: (name, vocab, hidden, batch, dtype, seed, mask recipe, extra mask words)
# inputs come from oracle.kernel_case_inputs (seeded); only outputs and input hashes are stored
# ---------------------------------------------------------------------------
SPARSE_CASES = [
    ("v1000_h256_b3_f16_mixed", 1000, 256, 3, "float16", 11, "u50+zero+full", 0),
    ("v1000_h256_b1_f16_random", 1000, 256, 1, "float16", 12, "random", 0),
    ("v4096_h512_b1_bf16_k13", 4096, 512, 1, "bfloat16", 13, "u13", 0),
    ("v4096_h512_b1_f16_k1", 4096, 512, 1, "float16", 14, "u1", 0),
    ("v2048_h128_b1_f16_wide", 2048, 128, 1, "float16", 15, "u300", 5),
    ("v777_h96_b2_f16_clustered", 777, 96, 2, "float16", 16, "c200+u3", 0),
    ("v3000_h264_b4_bf16_mixed", 3000, 264, 4, "bfloat16", 17, "c64+random+first+u700", 0),
]

BLOCK_CASES = [
    ("v1000_h256_b2_f16_mixed", 1000, 256, 2, "float16", 21, "u7+u400", 0),
    # fp16 only: the Triton CPU interpreter's tl.dot multiplies bf16 operands as raw
    # integer bit patterns, so bf16 block-GEMM outputs are pinned by the dense-mask fixture.
    ("v2048_h128_b5_f16", 2048, 128, 5, "float16", 22, "c40+first+zero+full+u100", 0),
    ("v1000_h64_b17_f16", 1000, 64, 17, "float16", 23, "u7+u300+random", 0),
    ("v4096_h512_b4_f16_sparse", 4096, 512, 4, "float16", 24, "c30+c30+u7+u2", 0),
]


def run_sparse_kernel(h, w, mask):
    vocab, hidden = w.shape
    batch = h.shape[0]
    mask_words = (vocab + 31) // 32
    out = torch.empty((batch, vocab), dtype=h.dtype)
    grid = (batch, (vocab + 31) // 32)
    ref_tr._bitmask_sparse_lm_head_kernel[grid](
        h, w, torch.from_numpy(mask), out,
        VOCAB=vocab, HIDDEN=hidden, MASK_WORDS=mask_words, BLOCK_M=32, BLOCK_K=256, num_warps=4)
    return out


def run_block_kernel(h, w, mask):
    vocab, hidden = w.shape
    batch = h.shape[0]
    mask_words = (vocab + 31) // 32
    out = torch.empty((batch, vocab), dtype=h.dtype)
    grid = ((batch + 15) // 16, (vocab + 31) // 32)
    ref_tr._bitmask_block_gemm_kernel[grid](
        h, w, torch.from_numpy(mask), out,
        BATCH=batch, VOCAB=vocab, HIDDEN=hidden, MASK_WORDS=mask_words,
        BLOCK_M=16, BLOCK_N=32, BLOCK_K=64, num_warps=4, num_stages=3)
    return out


def run_dense_mask(h, w, mask):
    logits = torch.nn.functional.linear(h.float(), w.float()).to(h.dtype)  # fp32 accumulate, one rounding
    batch, vocab = logits.shape
    xgr.apply_token_bitmask_inplace(logits, torch.from_numpy(mask).reshape(batch, -1),
                                    vocab_size=vocab, backend="cpu")
    return logits


def kernel_fixture(cases, runner, path):
    arrays, meta = {}, []
    for name, vocab, hidden, batch, dtype, seed, recipe, extra in cases:
        w, h, mask = O.kernel_case_inputs(vocab, hidden, batch, dtype, seed, recipe, extra)
        if runner is run_sparse_kernel and extra and batch > 1:
            raise AssertionError("wide masks with batch > 1 hit the reference's fixed-stride quirk")
        out = runner(h, w, mask)
        arrays[f"{name}/out"] = bits16(out)
        meta.append({"name": name, "vocab": vocab, "hidden": hidden, "batch": batch,
                     "dtype": dtype, "seed": seed, "recipe": recipe, "extra_words": extra,
                     "weight_sha256": O.tensor_sha256(w), "hidden_sha256": O.tensor_sha256(h),
                     "mask_sha256": O.tensor_sha256(mask)})
    arrays["meta"] = np.array(json.dumps(meta))
    np.savez_compressed(path, **arrays)
    print("wrote", path, len(meta), "cases")


# ---------------------------------------------------------------------------
# constrained_projection
# ---------------------------------------------------------------------------
def projection_fixture(path):
    arrays, meta = {}, []
    cases = []
    # The 32,768 x 1,024 fp32, batch-1, 1% uniform configuration (seed 0).
    w, h, ids = O.config0_inputs(seed=0)
    cases.append(("config0_fp32_1pct", w, h, torch.from_numpy(ids), 0.30, 0))
    for dt, seed in (("float16", 31), ("bfloat16", 32)):
        w2, h2 = O.projection_case_inputs(dt, seed)
        rng = np.random.default_rng(seed + 1000)
        dup = torch.from_numpy(rng.integers(0, 3000, size=50))
        dup = torch.cat([dup, dup[:10]])  # duplicates collapse
        cases.append((f"small_{dt}_dups_sparse", w2, h2, dup, 0.30, seed))
        dense_ids = torch.from_numpy(rng.choice(3000, size=1200, replace=False))
        cases.append((f"small_{dt}_dense_selected", w2, h2, dense_ids, 0.30, seed))
        cases.append((f"small_{dt}_unconstrained", w2, h2[0], None, 0.30, seed))
    for name, w, h, ids, thr, seed in cases:
        res = ref_runtime.constrained_projection(h, w, ids, dense_threshold=thr)
        entry = {"name": name, "mode": res.mode, "threshold": thr, "dtype": str(w.dtype).replace("torch.", ""),
                 "seed": seed, "weight_sha256": O.tensor_sha256(w), "hidden_sha256": O.tensor_sha256(h),
                 "hidden_1d": h.ndim == 1, "ids_is_none": ids is None}
        if ids is not None:
            arrays[f"{name}/ids"] = ids.numpy()
        arrays[f"{name}/token_ids"] = res.token_ids.numpy()
        lg = res.logits
        arrays[f"{name}/logits"] = bits16(lg) if lg.dtype != torch.float32 else lg.numpy()
        meta.append(entry)
    # error behaviour (gsp/runtime.py:35-40)
    errors = {}
    w = torch.zeros((100, 8))
    h = torch.zeros((1, 8))
    for label, ids in (("empty", torch.zeros(0, dtype=torch.long)),
                       ("negative", torch.tensor([-1, 3])),
                       ("too_large", torch.tensor([5, 100])),
                       ("two_dim", torch.tensor([[1, 2]]))):
        try:
            ref_runtime.constrained_projection(h, w, ids)
            errors[label] = None
        except ValueError as exc:
            errors[label] = str(exc)
    arrays["errors"] = np.array(json.dumps(errors))
    arrays["meta"] = np.array(json.dumps(meta))
    np.savez_compressed(path, **arrays)
    print("wrote", path, len(meta), "cases")


# ---------------------------------------------------------------------------
# routes and full-word fraction
# ---------------------------------------------------------------------------
def routes_fixture(path):
    calls = []

    def rec(name):
        def f(*args, **kwargs):
            calls.append(name)
            return torch.zeros(1)
        return f

    orig = (ref_tr.dense_masked_logits, ref_tr.bitmask_sparse_logits, ref_tr.bitmask_block_gemm_logits)
    ref_tr.dense_masked_logits = rec("dense")
    ref_tr.bitmask_sparse_logits = rec("row")
    ref_tr.bitmask_block_gemm_logits = rec("block")
    out = {"dispatch_cases": [], "grid": [], "full_word_fraction": []}
    try:
        vocab, hidden = 8192, 512
        words = (vocab + 31) // 32
        plan = [(1, "all_sparse"), (1, "all_dense")]
        for b in (2, 4, 8, 16, 32):
            plan += [(b, "all_sparse"), (b, "all_dense"), (b, "mixed")]
        for batch, pattern in plan:
            mask = torch.zeros((batch, words), dtype=torch.int32)
            for i in range(batch):
                if pattern == "all_dense" or (pattern == "mixed" and i % 2):
                    mask[i].fill_(-1)
                else:
                    mask[i, 0] = 1
            frac = ref_tr.full_word_fraction_cpu(mask)
            h = torch.zeros((batch, hidden)) if batch > 1 else torch.zeros((1, hidden))
            _, route = ref_tr.adaptive_grammar_logits(h, None, None, full_word_fraction=frac)
            _, route_none = ref_tr.adaptive_grammar_logits(h, None, None)
            out["dispatch_cases"].append({"batch": batch, "pattern": pattern, "fwf": frac,
                                          "route": route, "route_without_fwf": route_none})
        rng = np.random.default_rng(41)
        for _ in range(300):
            batch = int(rng.choice([1, 2, 3, 8, 31, 32, 33, 64]))
            frac = [float(x) for x in rng.choice([0.0, 0.1, 0.24, 0.25, 0.26, 0.79, 0.8, 0.81, 1.0], size=batch)]
            thr = float(rng.choice([0.5, 0.8, 0.9]))
            h = torch.zeros((batch, 4))
            _, route = ref_tr.adaptive_grammar_logits(h, None, None, full_word_fraction=frac,
                                                      dense_full_word_threshold=thr)
            out["grid"].append({"batch": batch, "fwf": frac, "threshold": thr, "route": route})
        for seed in range(6):
            r2 = np.random.default_rng(100 + seed)
            batch = int(r2.integers(1, 5))
            width = int(r2.integers(1, 40))
            m = r2.integers(-2**31, 2**31 - 1, size=(batch, width), dtype=np.int64).astype(np.int32)
            m[:, r2.random(width) < 0.4] = -1
            out["full_word_fraction"].append({"mask": m.tolist(),
                                              "fwf": ref_tr.full_word_fraction_cpu(torch.from_numpy(m))})
    finally:
        ref_tr.dense_masked_logits, ref_tr.bitmask_sparse_logits, ref_tr.bitmask_block_gemm_logits = orig
    with open(path, "w") as f:
        json.dump(out, f, indent=1)
    print("wrote", path)


def main():
    kernel_fixture(SPARSE_CASES, run_sparse_kernel, os.path.join(HERE, "row_sparse_ref.npz"))
    kernel_fixture(BLOCK_CASES, run_block_kernel, os.path.join(HERE, "block_gemm_ref.npz"))
    kernel_fixture(SPARSE_CASES + BLOCK_CASES, run_dense_mask, os.path.join(HERE, "dense_mask_ref.npz"))
    projection_fixture(os.path.join(HERE, "projection_ref.npz"))
    routes_fixture(os.path.join(HERE, "routes_ref.json"))


if __name__ == "__main__":
    main()
