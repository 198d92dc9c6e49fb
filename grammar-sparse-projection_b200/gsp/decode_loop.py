"""Grammar-constrained decode loop around the B200 head: the integration of the
reference's decode loops (benchmarks/qwen35_adaptive_paired.py:46-110) with
this library as the drop-in LM head.

Per step, as the reference does it:
  1. the grammar matcher fills the request's packed bitmask in pinned host
     memory (xgrammar GrammarMatcher.fill_next_token_bitmask);
  2. the host computes the full-word fraction (full_word_fraction_cpu) for
     the reference dispatch rule;
  3. the mask is copied to the device (copy_bitmask_to_gpu, non-blocking);
  4. the model produces the last hidden state of each request;
  5. the head projects it (adaptive_grammar_logits with the reference's
     signature, or the dense route, or the fused greedy top-1, or the
     CUDA-graphed head with its device-side route choice);
  6. the next token is taken (teacher-forced target or greedy argmax) and
     given to the matcher (accept_token), which must accept it.

The reference drives Qwen3.5-2B from Hugging Face. Any model works here: the
loop needs only `step(tokens) -> hidden [B, H]` and the LM-head weight
[V, H]. TinyDecoder is a small seeded stand-in (embedding, residual MLP
blocks, RMSNorm) for machines without the checkpoint, and SyntheticVocabulary
a token list with a greedy longest-match tokenizer, from which xgrammar builds
its TokenizerInfo without network access.
"""
from __future__ import annotations

import dataclasses
import json
import time

import torch

from . import triton_runtime as tr
from .graphed import GraphedGrammarHead


class SyntheticVocabulary:
    """Token strings for a vocabulary of `size` tokens: id 0 is the stop token,
    then every printable ASCII character (so any ASCII text is encodable),
    then JSON punctuation pieces and the caller's extra pieces, then filler
    tokens "<f{i}>" up to `size`."""

    JSON_PIECES = ('{"', '":', '",', '"}', '":"', '","', '":{"', '"}}', '":[', '],"', 'true', 'false', 'null',
                   '"]', '["', '":true', '":false', '":0', '":1', '":2', '":3', '":4', '":5')

    def __init__(self, size: int, extra_pieces: tuple[str, ...] = ()):
        tokens = ["</s>"] + [chr(c) for c in range(32, 127)]
        seen = set(tokens)
        for piece in self.JSON_PIECES + tuple(extra_pieces):
            if piece not in seen:
                tokens.append(piece)
                seen.add(piece)
        if size < len(tokens):
            raise ValueError(f"vocabulary size {size} is below the {len(tokens)} base tokens")
        tokens += [f"<f{i}>" for i in range(size - len(tokens))]
        self.tokens = tokens
        self.index = {t: i for i, t in enumerate(tokens)}
        self.max_len = max(len(t) for t in tokens[1:128 + len(extra_pieces) + len(self.JSON_PIECES)])
        self.stop_id = 0

    def __len__(self) -> int:
        return len(self.tokens)

    def encode(self, text: str) -> list[int]:
        """Greedy longest match (every ASCII character is a token)."""
        out, i = [], 0
        while i < len(text):
            for n in range(min(self.max_len, len(text) - i), 0, -1):
                tid = self.index.get(text[i:i + n])
                if tid is not None and not self.tokens[tid].startswith("<f"):
                    out.append(tid)
                    i += n
                    break
            else:
                raise ValueError(f"character {text[i]!r} is not in the vocabulary")
        return out

    def decode(self, ids) -> str:
        return "".join("" if i == self.stop_id else self.tokens[i] for i in ids)

    def tokenizer_info(self):
        import xgrammar as xgr
        return xgr.TokenizerInfo(self.tokens, vocab_type=xgr.VocabType.RAW, stop_token_ids=[self.stop_id])


class TinyDecoder(torch.nn.Module):
    """Seeded stand-in for a decoder-only transformer: token embedding plus a
    position embedding, `layers` pre-norm residual MLP blocks and a final
    RMSNorm. step(tokens [B]) returns the next hidden states [B, H] and
    advances each request's position (the state a KV cache would hold)."""

    def __init__(self, vocab: int, hidden: int, *, layers: int = 2, max_positions: int = 4096, seed: int = 0,
                 dtype: torch.dtype = torch.float16, device="cuda"):
        super().__init__()
        g = torch.Generator(device="cpu").manual_seed(seed)
        def param(*shape, scale):
            return torch.nn.Parameter((torch.randn(*shape, generator=g) * scale).to(device=device, dtype=dtype),
                                      requires_grad=False)
        self.embed = param(vocab, hidden, scale=1.0)
        self.pos = param(max_positions, hidden, scale=0.5)
        self.up = torch.nn.ParameterList([param(hidden, 2 * hidden, scale=hidden ** -0.5) for _ in range(layers)])
        self.down = torch.nn.ParameterList([param(2 * hidden, hidden, scale=(2 * hidden) ** -0.5)
                                            for _ in range(layers)])
        self.position = None

    @staticmethod
    def _rms(x):
        return x * torch.rsqrt(x.float().pow(2).mean(-1, keepdim=True) + 1e-6).to(x.dtype)

    def reset(self, batch: int):
        self.position = torch.zeros(batch, dtype=torch.long, device=self.embed.device)

    @torch.inference_mode()
    def step(self, tokens: torch.Tensor) -> torch.Tensor:
        x = self.embed[tokens] + self.pos[self.position.clamp_max(self.pos.shape[0] - 1)]
        for up, down in zip(self.up, self.down):
            x = x + torch.nn.functional.gelu(self._rms(x) @ up) @ down
        self.position += 1
        return self._rms(x).contiguous()


@dataclasses.dataclass
class StepRecord:
    step: int
    tokens: list[int]
    routes: str
    full_word_fraction: list[float]
    head_us: float


HEAD_MODES = ("adaptive", "dense", "fused-top1", "graphed")


class GrammarDecodeLoop:
    """Batched grammar-constrained decoding with one xgrammar matcher per
    request and this library's head. `model` has reset(batch) and
    step(tokens [B] on the device) -> hidden [B, H]; `weight` is the LM head
    [V, H]; `vocab` a SyntheticVocabulary (or any object with tokenizer_info()
    and stop_id)."""

    def __init__(self, model, weight: torch.Tensor, vocab, *, head: str = "adaptive", policy: str = "reference"):
        import xgrammar as xgr
        if head not in HEAD_MODES:
            raise ValueError(f"head must be one of {HEAD_MODES}")
        self.model, self.weight, self.vocab = model, weight, vocab
        self.head, self.policy = head, policy
        self.compiler = xgr.GrammarCompiler(vocab.tokenizer_info())
        self._graphed = None

    def new_matchers(self, schemas) -> list:
        import xgrammar as xgr
        return [xgr.GrammarMatcher(self.compiler.compile_json_schema(
            s if isinstance(s, str) else json.dumps(s))) for s in schemas]

    def _project(self, hidden: torch.Tensor, mask_cpu: torch.Tensor, mask_gpu: torch.Tensor, fractions):
        """Returns (logits [B, V] or None, next greedy tokens [B] on the device, route string)."""
        if self.head == "graphed":  # mask_cpu is the head's own pinned staging buffer
            head = self._graphed
            head.stage_mask()
            out = head.step(hidden)
            return out.logits, out.top_index, tr.ROUTES[int(out.route.item())]
        tr.copy_bitmask_to_gpu(mask_cpu, mask_gpu)
        if self.head == "dense":
            logits = tr.dense_masked_logits(hidden, self.weight, mask_gpu)
            return logits, logits.argmax(-1), "dense-mask"
        if self.head == "fused-top1":
            route = tr._reference_route(hidden.shape[0], fractions, 0.80)
            logits, _, top_index = tr.grammar_logits_with_top1(hidden, self.weight, mask_gpu, route=route)
            return logits, top_index, route
        logits, route = tr.adaptive_grammar_logits(hidden, self.weight, mask_gpu, full_word_fraction=fractions,
                                                   policy=self.policy)
        logits = logits.reshape(hidden.shape[0], -1)
        return logits, logits.argmax(-1), route

    def run(self, schemas, *, targets: list[list[int]] | None = None, max_steps: int = 64, on_step=None):
        """Decodes one request per schema. With `targets` (token ids per
        request) the loop is teacher-forced, as the reference's is; without,
        it takes the greedy token. Finished requests (matcher terminated) keep
        an all-legal mask and are not advanced. on_step(step, hidden, mask_cpu,
        logits, tokens, route) is called before the tokens are accepted.
        Returns (token ids per request, list of StepRecord)."""
        batch = len(schemas)
        matchers = self.new_matchers(schemas)
        vocab = self.weight.shape[0]
        if self.head == "graphed":
            if self._graphed is None or self._graphed.batch != batch:
                self._graphed = GraphedGrammarHead(self.weight, batch)
            mask_cpu = self._graphed.mask_host
        else:
            mask_cpu = tr.allocate_pinned_bitmask(batch, vocab)
        mask_gpu = torch.empty(mask_cpu.shape, dtype=torch.int32, device=self.weight.device)
        self.model.reset(batch)
        out = [[] for _ in range(batch)]
        done = [False] * batch
        records = []
        prev = torch.full((batch,), self.vocab.stop_id, dtype=torch.long, device=self.weight.device)
        steps = max(len(t) for t in targets) if targets is not None else max_steps
        for step in range(steps):
            if self.head == "graphed":
                self._graphed.wait_mask_copied()  # the last staged copy has read the buffer
            for b, m in enumerate(matchers):
                if done[b] or (targets is not None and step >= len(targets[b])):
                    mask_cpu[b].fill_(-1)
                else:
                    m.fill_next_token_bitmask(mask_cpu, b)
            fractions = tr.full_word_fraction_cpu(mask_cpu)
            hidden = self.model.step(prev)
            t0 = time.perf_counter()
            logits, greedy, route = self._project(hidden, mask_cpu, mask_gpu, fractions)
            greedy = greedy.tolist()
            head_us = (time.perf_counter() - t0) * 1e6
            tokens = []
            for b in range(batch):
                if targets is not None:
                    tokens.append(targets[b][step] if step < len(targets[b]) else self.vocab.stop_id)
                else:
                    tokens.append(int(greedy[b]))
            if on_step is not None:
                on_step(step, hidden, mask_cpu, logits, greedy, route)
            for b, m in enumerate(matchers):
                if done[b] or (targets is not None and step >= len(targets[b])):
                    continue
                if not m.accept_token(tokens[b]):
                    raise RuntimeError(f"request {b}: the matcher rejected token {tokens[b]} at step {step}")
                out[b].append(tokens[b])
                if m.is_terminated():
                    done[b] = True
            records.append(StepRecord(step, tokens, route, list(fractions), head_us))
            prev = torch.tensor(tokens, dtype=torch.long, device=self.weight.device)
            if all(done):
                break
        return out, records
