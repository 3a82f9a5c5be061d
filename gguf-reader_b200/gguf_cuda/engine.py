"""Engine: the generate / chat loops of src/infer/engine.rs over the device model.

The loops are host logic in the reference too; here they drive LlamaModel with
the logits left on the device and sampled there (ggc_model_sample), so a step
returns one token id.  Tokenizing and UTF-8 streaming stay with the caller:
``encode(text) -> ids`` is passed in, and the loops work on token ids.

  * ``generate`` (engine.rs:74-138): forward the prompt at positions 0.. (on top
    of whatever the cache holds, as the reference's forward does), then sample ->
    record -> forward(1 token) at positions that continue from the prompt,
    until EOS or max_tokens.
  * ``chat`` (engine.rs:255-378): the Qwen2 chat template (system prompt on the
    first turn), an incremental forward of the NEW tokens only at positions that
    continue from the cache (the history's K/V are reused), the repeat-penalty
    history rebuilt from the previous turns, and the im_end token forwarded after
    the reply; ``reset`` clears the cache, the sampler history and the chat state
    (engine.rs:516-521).
  * The sampler's RNG stays here: ``draw()`` returns the uniform the reference's
    StdRng would give (a seeded numpy generator by default).
  * Configurations that keep more than 1024 candidates after top-k (top_k = 0
    or above 1024) are sampled on the host from the logits of the last forward
    (``sampling.sample_host``), since the device kernel holds at most 1024.
"""
from __future__ import annotations

from collections import Counter
from typing import Callable

import numpy as np

from .sampling import device_can_sample, sample_host

IM_START, IM_END, TOK_USER, TOK_ASSISTANT, TOK_SYSTEM = 151644, 151645, 872, 77091, 8948
SYSTEM_PROMPT = "You are a helpful assistant."
DEFAULT_SAMPLER = dict(temperature=1.0, top_k=40, top_p=0.95, min_p=0.0, repeat_penalty=1.1)   # sampler.rs:28-37


class Engine:
    def __init__(self, model, encode: Callable[[str], list], eos: int | None = None, sampler: dict | None = None,
                 draw: Callable[[], float] | None = None, seed: int = 0, context_length: int | None = None,
                 decode: Callable[[list], str] | None = None):
        self.model = model
        self.encode = encode
        self.decode = decode   # when given, a reply is re-encoded from its text for the history, as the reference does
        self.eos = eos
        self.sampler = dict(DEFAULT_SAMPLER, **(sampler or {}))
        rng = np.random.default_rng(seed)
        self.draw = draw or (lambda: float(np.float32(rng.random())) % 1.0)
        self.context_length = context_length
        self.seen = Counter()          # Sampler::record counts (sampler.rs:80-83)
        self.chat_prefilled = False
        self.chat_history = []         # (user text, reply ids)
        self.host_sampling = not device_can_sample(self.sampler, model.vocab)
        self._logits = None

    def _forward(self, ids, pos):
        out = self.model.forward(ids, pos, want_logits=self.host_sampling)
        if self.host_sampling:
            self._logits = out

    # Sampler::sample over the model's last logits (on the device unless it keeps > 1024 candidates)
    def _sample(self) -> int:
        seen = [t for t, c in self.seen.items() if c > 0]
        if self.host_sampling:
            return sample_host(self._logits, self.sampler, seen, self.draw())
        return self.model.sample(self.sampler, seen, self.draw())

    def _loop(self, max_tokens: int, pos=None) -> list:
        out = []
        for _ in range(max_tokens):
            tid = self._sample()
            if self.eos is not None and tid == self.eos:
                break
            out.append(tid)
            self.seen[tid] += 1
            p = self.model.cache_len() if pos is None else pos
            self._forward([tid], [p])
            if pos is not None:
                pos += 1
        return out

    def generate(self, prompt_ids, max_tokens: int) -> list:
        """engine.rs:74-138 over token ids (the prompt from position 0)."""
        ids = [int(t) for t in prompt_ids]
        if not ids:
            raise ValueError("prompt tokenize empty")
        self._forward(ids, list(range(len(ids))))
        return self._loop(max_tokens, pos=len(ids))

    def chat(self, text: str, max_tokens: int) -> list:
        """engine.rs:255-378: one turn; returns the reply's token ids."""
        nl = list(self.encode("\n"))
        new = []
        if not self.chat_prefilled:
            new += [IM_START, TOK_SYSTEM] + nl + list(self.encode(SYSTEM_PROMPT)) + [IM_END] + nl
        new += [IM_START, TOK_USER] + nl + list(self.encode(text)) + [IM_END] + nl + [IM_START, TOK_ASSISTANT] + nl
        self.chat_prefilled = True
        limit = self.context_length
        if limit is not None and self.model.cache_len() + len(new) > limit:
            raise ValueError(f"context exceeded: {self.model.cache_len()} + {len(new)} > {limit}")
        start = self.model.cache_len()
        self._forward(new, list(range(start, start + len(new))))   # only the new tokens
        self.seen = Counter()                                   # sampler.reset() then the history (:325-334)
        for user, reply in self.chat_history:
            self.seen.update(int(t) for t in self.encode(user))
            self.seen.update(int(t) for t in self.encode(self.decode(reply))) if self.decode else self.seen.update(reply)
        out = self._loop(max_tokens)
        self.chat_history.append((text, out))
        self.model.forward([IM_END], [self.model.cache_len()], want_logits=False)   # close the reply (:372-375)
        return out

    def reset(self):
        self.model.reset_cache()
        self.seen = Counter()
        self.chat_prefilled = False
        self.chat_history = []
