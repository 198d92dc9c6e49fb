"""The decode loop (benchmarks/qwen35_adaptive_paired.py:46-110 of the
reference) run through this library's head: an xgrammar matcher per request
fills a pinned mask each step, the full-word fraction feeds the reference
dispatch rule, the mask goes to the device, a model produces the hidden state,
the head projects it and the next token goes back to the matcher.

Offline stand-ins: a 32,768-token synthetic vocabulary (every printable ASCII
character plus JSON pieces and fillers) from which xgrammar builds its
TokenizerInfo, and a seeded tiny decoder in place of the transformer. At every
step the head's output is checked against the oracle on that step's hidden
state and mask: legal support bit-exact, values within the fp16 tolerance,
the route equal to the reference rule's, the next token (greedy) equal to the
exact argmax except within the near-tie window, and the matcher accepting it.
"""
import json

import numpy as np
import pytest
import torch

from gsp import triton_runtime as tr
from gsp.decode_loop import GrammarDecodeLoop, SyntheticVocabulary, TinyDecoder
from oracle import gsp_oracle as O

pytestmark = pytest.mark.gpu

VOCAB, HIDDEN = 32_768, 512

CASES = [
    ({"type": "object",
      "properties": {"unit": {"enum": ["kg", "lb", "oz"]},
                     "count": {"type": "integer", "minimum": 0, "maximum": 99},
                     "fragile": {"type": "boolean"}},
      "required": ["unit", "count", "fragile"], "additionalProperties": False},
     '{"unit":"lb","count":42,"fragile":false}'),
    ({"type": "object",
      "properties": {"op": {"const": "resize"},
                     "args": {"type": "object",
                              "properties": {"width": {"type": "integer"}, "height": {"type": "integer"},
                                             "keep_ratio": {"type": "boolean"}},
                              "required": ["width", "height", "keep_ratio"], "additionalProperties": False}},
      "required": ["op", "args"], "additionalProperties": False},
     '{"op":"resize","args":{"width":640,"height":480,"keep_ratio":true}}'),
    ({"type": "object",
      "properties": {"note": {"type": "string", "maxLength": 24},
                     "tags": {"type": "array", "items": {"enum": ["red", "green", "blue"]}, "maxItems": 3}},
      "required": ["note", "tags"], "additionalProperties": False},
     '{"note":"ship by friday","tags":["red","blue"]}'),
]


@pytest.fixture(scope="module")
def setup(cuda_device):
    vocab = SyntheticVocabulary(VOCAB, extra_pieces=("unit", "count", "fragile", "resize", "width", "height"))
    g = torch.Generator(device="cpu").manual_seed(11)
    w = (torch.randn(VOCAB, HIDDEN, generator=g) * 0.02).half()
    model = TinyDecoder(VOCAB, HIDDEN, seed=3, device=cuda_device)
    return vocab, w, w.to(cuda_device), model


def _checker(w_cpu, batch, seen):
    def on_step(step, hidden, mask_cpu, logits, greedy, route):
        mask = mask_cpu.numpy().copy()
        exact = O.masked_logits_exact(hidden.cpu(), w_cpu, mask)
        got = logits.reshape(batch, -1).cpu()
        rep = O.compare_logits(exact, got, dtype=torch.float16)
        assert rep["support"] and rep["values"], (step, rep)
        assert O.top1_agrees(exact, torch.tensor(greedy), dtype=torch.float16), step
        seen.append(route)
    return on_step


@pytest.mark.parametrize("head", ["adaptive", "fused-top1"])
def test_teacher_forced_single_requests(setup, head):
    vocab, w_cpu, w, model = setup
    loop = GrammarDecodeLoop(model, w, vocab, head=head)
    routes = []
    for schema, sample in CASES:
        targets = vocab.encode(sample) + [vocab.stop_id]
        out, records = loop.run([schema], targets=[targets], on_step=_checker(w_cpu, 1, routes))
        assert vocab.decode(out[0]) == sample
        assert len(records) == len(targets)
        for rec in records:  # the reference rule on this step's full-word fraction
            assert rec.routes == O.adaptive_route(1, rec.full_word_fraction), rec
    # the reference rule sends batch 1 to row-sparse whatever the density
    # (its dense fallback needs batch > 1, gsp/triton_runtime.py:346)
    assert set(routes) == {"row-sparse"}, routes


def test_teacher_forced_batch_of_three(setup):
    vocab, w_cpu, w, model = setup
    loop = GrammarDecodeLoop(model, w, vocab, head="adaptive")
    targets = [vocab.encode(s) + [vocab.stop_id] for _, s in CASES]
    routes = []
    out, records = loop.run([c for c, _ in CASES], targets=targets, on_step=_checker(w_cpu, 3, routes))
    for b, (_, sample) in enumerate(CASES):
        assert vocab.decode(out[b]) == sample
    for rec in records:
        assert rec.routes == O.adaptive_route(3, rec.full_word_fraction), rec
    assert set(routes) <= {"block-sparse", "dense-mask"}


@pytest.mark.parametrize("head", ["adaptive", "fused-top1", "graphed", "dense"])
def test_free_running_greedy_batch(setup, head):
    """Greedy decoding: every token the head picks is legal (the matcher
    accepts it) and equals the oracle's argmax on that step's inputs."""
    vocab, w_cpu, w, model = setup
    loop = GrammarDecodeLoop(model, w, vocab, head=head)
    routes = []
    out, records = loop.run([c for c, _ in CASES], max_steps=48, on_step=_checker(w_cpu, 3, routes))
    assert len(records) >= 4
    for b in range(3):
        assert len(out[b]) >= 1
        text = vocab.decode(out[b])
        if records[-1].step < 47:  # every request finished: its text is valid JSON of its schema
            obj = json.loads(text)
            assert set(obj) == set(CASES[b][0]["required"])
