"""Stand-ins for the target model and tokenizer of ``batch_generate``.

The reference's loop (hsd/dots_ocr_pipeline/modeling_dots_ocr_hsd.py
``DotsOCRForCausalLM.batch_generate``, D:923-1810) touches its model only
through ``self.model.config._attn_implementation`` (D:948-949) and
``self.forward(**model_inputs)`` -> ``.logits`` / ``.past_key_values``
(D:1059-1064, D:1603), and compacts the returned cache with
``index_select(-2, keep)`` on every layer's keys and values (D:1704-1722).
Its tokenizer use is ``encode`` / ``decode`` / ``batch_decode`` /
``pad_token_id`` and, for the page block's candidate trees, a pre-tokenizer
called on a list of strings (D:628-745).  The classes here provide exactly
that, deterministically, so the unmodified loop can run on the CPU (to
record golden traces) and the package's drop-in can run on the same model
(to be checked against them).

* :class:`CharTokenizer` -- one token per character of a small alphabet.
* :class:`StandInLM` -- a "true text" model: each block (identified by the
  first tokens of its prompt) has a target text; a row whose visible context
  (the tokens of the KV columns it sees, in column order) continues the
  block's prompt with a prefix of its text predicts the next character
  (EOS at the end), any other row a token hashed from its last context
  tokens.  Its cache stores, per KV column, the token, a running column id
  and the position, so a trace of the cache after compaction shows exactly
  which columns were kept.
"""
from __future__ import annotations

import hashlib
from types import SimpleNamespace

import numpy as np
import torch

PAD, EOS = 0, 1
_ALPHABET = [chr(c) for c in range(32, 127)] + ["\n"]
_FIRST = 4                                  # ids 0-3: specials
VOCAB = _FIRST + len(_ALPHABET)


class CharTokenizer:
    """Character-level tokenizer (printable ASCII and newline)."""

    pad_token_id = PAD
    eos_token_id = EOS

    def __init__(self):
        self._ids = {c: _FIRST + i for i, c in enumerate(_ALPHABET)}

    def encode(self, text, add_special_tokens=False):
        return [self._ids[c] for c in text if c in self._ids]

    def __call__(self, texts, add_special_tokens=False):
        if isinstance(texts, str):
            return {"input_ids": self.encode(texts)}
        return {"input_ids": [self.encode(t) for t in texts]}

    def decode(self, ids, skip_special_tokens=False):
        if isinstance(ids, (int, np.integer)):
            ids = [int(ids)]
        return "".join(_ALPHABET[i - _FIRST] for i in map(int, ids) if i >= _FIRST)

    def batch_decode(self, seqs, skip_special_tokens=True):
        return [self.decode(s) for s in seqs]


class _Layer:
    def __init__(self, t):
        self.keys = t
        self.values = t.clone()


class StandInCache:
    """One layer whose keys / values rows are (token, column id, position, 0)
    per KV column (int64, ``[1, 1, KV, 4]``): compaction by
    ``index_select(-2, keep)`` keeps them aligned with the mask's columns."""

    def __init__(self, device):
        self.layers = [_Layer(torch.zeros((1, 1, 0, 4), dtype=torch.int64, device=device))]
        self.next_id = 0

    def append(self, tokens, positions):
        n = tokens.numel()
        rows = torch.stack([tokens.reshape(-1).long(),
                            torch.arange(self.next_id, self.next_id + n, device=tokens.device),
                            positions.reshape(-1).long(),
                            torch.zeros(n, dtype=torch.long, device=tokens.device)], 1)
        self.next_id += n
        lay = self.layers[0]
        lay.keys = torch.cat([lay.keys, rows[None, None]], dim=-2)
        lay.values = torch.cat([lay.values, rows[None, None]], dim=-2)

    def columns(self):
        return self.layers[0].keys[0, 0].cpu().numpy()


def _allowed_from_mask(attention_mask, q, kv):
    """Dense bool ``[q, kv]`` from the reference's float mask or a mask
    object of the package (anything with ``.plan().dense_allowed()``)."""
    if isinstance(attention_mask, torch.Tensor):
        m = attention_mask
        while m.dim() > 2:
            m = m[0]
        return (m[:, :kv] > -0.1).cpu().numpy()
    return attention_mask.plan().dense_allowed()[:q, :kv]


class StandInLM:
    """Deterministic target model (see the module docstring).  ``prompts[b]``
    and ``texts[b]`` are block b's prompt and target text (token lists);
    ``trace`` records every forward's inputs."""

    def __init__(self, prompts, texts, vocab=VOCAB, eos=EOS, head=6, graded=False):
        self.model = SimpleNamespace(config=SimpleNamespace(_attn_implementation="eager"))
        self.heads = {tuple(int(t) for t in p[:head]): b for b, p in enumerate(prompts)}
        self.prompts = [list(map(int, p)) for p in prompts]
        self.texts = [list(map(int, t)) for t in texts]
        self.vocab, self.eos, self.head = vocab, eos, head
        self.graded = graded
        self.trace = []

    def predict(self, ctx):
        b = self.heads.get(tuple(int(t) for t in ctx[:self.head]))
        if b is not None and len(ctx) >= len(self.prompts[b]):
            gen = ctx[len(self.prompts[b]):]
            text = self.texts[b]
            if len(gen) <= len(text) and list(gen) == text[:len(gen)]:
                return text[len(gen)] if len(gen) < len(text) else self.eos
        h = 0
        for t in ctx[-3:]:
            h = (h * 1000003 + int(t) + 7) % 2147483647
        return _FIRST + h % (self.vocab - _FIRST)

    def forward(self, input_ids=None, attention_mask=None, position_ids=None,
                past_key_values=None, use_cache=True, **kwargs):
        dev = input_ids.device
        if past_key_values is None:
            past_key_values = StandInCache(dev)
        before = past_key_values.columns()
        if position_ids.dim() == 3:        # HunYuan's [1, 4, Q] positions: row 0
            position_ids = position_ids[:, 0]
        past_key_values.append(input_ids[0], position_ids[0])
        cols = past_key_values.columns()
        q, kv = input_ids.shape[1], cols.shape[0]
        allowed = _allowed_from_mask(attention_mask, q, kv)
        toks = cols[:, 0]
        pred = np.empty(q, dtype=np.int64)
        for r in range(q):
            pred[r] = self.predict(toks[allowed[r]].tolist())
        self.trace.append(dict(
            input_ids=input_ids[0].cpu().numpy().astype(np.int64),
            position_ids=position_ids[0].cpu().numpy().astype(np.int64),
            kept_column_ids=before[:, 1].astype(np.int64),
            mask_sha=hashlib.sha256(np.packbits(allowed, axis=-1).tobytes()
                                    + np.asarray(allowed.shape, np.int64).tobytes()).hexdigest()))
        if self.graded:
            rows = np.stack([self.graded_row(toks[allowed[r]].tolist(), int(pred[r]))
                             for r in range(q)]) if q else np.zeros((0, self.vocab), np.float32)
            logits = torch.from_numpy(rows)[None].to(torch.bfloat16)
        else:
            logits = torch.zeros((1, q, self.vocab), dtype=torch.float32)
            logits[0, torch.arange(q), torch.from_numpy(pred)] = 1.0
        return SimpleNamespace(logits=logits.to(dev), past_key_values=past_key_values)

    def graded_row(self, ctx, pred):
        """Logits of one row for the logit-ratio rules: 8 at the predicted
        token, every other token k / 8 with k in [0, 56] hashed from the last
        context tokens and the token (exact in bf16), so some draft tokens
        pass a ratio threshold below 1 without being the argmax."""
        h = 0
        for t in ctx[-2:]:
            h = (h * 1000003 + int(t) + 11) % 2147483647
        k = (h * 2654435761 + np.arange(self.vocab, dtype=np.int64) * 40503) % 57
        row = k.astype(np.float32) / 8.0
        row[pred] = 8.0
        return row

    __call__ = forward


def packed_prefill(prompts, device="cpu"):
    """The caller's packing of the reference (RD:232-245): every block's
    prompt one after another, positions restarting at 0 per block, a
    block-diagonal causal fp32 mask (0 / -inf) and ``pointer`` = cumulative
    ends - 1 (int64)."""
    lens = [len(p) for p in prompts]
    n = sum(lens)
    ids = torch.tensor([sum((list(map(int, p)) for p in prompts), [])], dtype=torch.long)
    pos = torch.cat([torch.arange(k) for k in lens])[None].long()
    allowed = torch.zeros((n, n), dtype=torch.bool)
    s = 0
    for k in lens:
        allowed[s:s + k, s:s + k] = torch.tril(torch.ones((k, k), dtype=torch.bool))
        s += k
    mask = torch.zeros((1, 1, n, n), dtype=torch.float32).masked_fill(~allowed[None, None],
                                                                      float("-inf"))
    pointer = torch.cumsum(torch.tensor(lens, dtype=torch.long), 0) - 1
    return (ids.to(device), mask.to(device), pos.to(device), pointer.to(device))


def _sha(a):
    a = np.ascontiguousarray(np.asarray(a, dtype=np.int64))
    return hashlib.sha256(a.tobytes()).hexdigest()[:20]


def step_digest(entry):
    """Compact, order-sensitive record of one forward: sizes and digests of
    the packed input ids, positions and kept KV column ids, and the mask
    digest (sha-256 prefixes; equal digests = bit-identical arrays)."""
    return dict(q=int(len(entry["input_ids"])), kv_kept=int(len(entry["kept_column_ids"])),
                ids=_sha(entry["input_ids"]), pos=_sha(entry["position_ids"]),
                kept=_sha(entry["kept_column_ids"]), mask=entry["mask_sha"][:20])


def oracle_model(lm):
    """``model(input_ids, position_ids, allowed, kv_tokens) -> next ids`` over
    the same rule as :meth:`StandInLM.forward`, for ``oracle.loop.reference_loop``."""
    def model(input_ids, position_ids, allowed, kv_tokens):
        kv_tokens = np.asarray(kv_tokens, dtype=np.int64)
        return np.asarray([lm.predict(kv_tokens[allowed[r]].tolist())
                           for r in range(allowed.shape[0])], dtype=np.int64)
    return model


def trace_digest(step):
    """:func:`step_digest` of one step of ``oracle.loop.reference_loop``'s trace."""
    allowed = np.asarray(step["allowed"], dtype=bool)
    sha = hashlib.sha256(np.packbits(allowed, axis=-1).tobytes()
                         + np.asarray(allowed.shape, np.int64).tobytes()).hexdigest()
    return step_digest(dict(input_ids=step["input_ids"], position_ids=step["position_ids"],
                            kept_column_ids=step["kept_column_ids"], mask_sha=sha))


def oracle_logits_model(lm):
    """Dense float32 logits ``[Q, V]`` of :meth:`StandInLM.graded_row` for
    ``oracle.loop.reference_loop(logits_model=...)``."""
    def fn(input_ids, position_ids, allowed, kv_tokens):
        kv_tokens = np.asarray(kv_tokens, dtype=np.int64)
        rows = []
        for r in range(allowed.shape[0]):
            ctx = kv_tokens[allowed[r]].tolist()
            rows.append(lm.graded_row(ctx, lm.predict(ctx)))
        return np.stack(rows).astype(np.float32)
    return fn
