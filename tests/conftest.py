import json
import os
import sys

import numpy as np
import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_ROOT = os.path.join(REPO, "grammar-sparse-projection_b200")
GOLDEN = os.path.join(REPO, "tests", "golden")
for p in (PKG_ROOT, REPO):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (B200) device")


def load_npz(name):
    data = np.load(os.path.join(GOLDEN, name), allow_pickle=False)
    meta = json.loads(str(data["meta"]))
    return data, meta


def load_json(name):
    with open(os.path.join(GOLDEN, name)) as f:
        return json.load(f)


@pytest.fixture(scope="session")
def cuda_device():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("GPU test collected on a machine without CUDA")
    return torch.device("cuda", 0)


def exact_logits_gpu(hidden, weight, mask, chunk_rows: int = 32768):
    """float64 masked logits of the same definition as the oracle's
    masked_logits_exact (dot products of the low-precision inputs, no rounding,
    -inf where illegal), computed on the GPU with plain torch for the
    full-size configurations the CPU oracle would take minutes over. Tests
    that use it also check it against the CPU oracle on sampled requests."""
    import torch
    batch, vocab = hidden.shape[0], weight.shape[0]
    h64 = hidden.double()
    out = torch.empty(batch, vocab, dtype=torch.float64, device=hidden.device)
    for r0 in range(0, vocab, chunk_rows):
        r1 = min(vocab, r0 + chunk_rows)
        out[:, r0:r1] = h64 @ weight[r0:r1].double().T
    v = torch.arange(vocab, device=hidden.device)
    legal = ((mask.reshape(batch, -1)[:, v >> 5] >> (v & 31)) & 1).bool()
    return out.masked_fill_(~legal, float("-inf"))
