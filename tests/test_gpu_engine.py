"""Engine (gguf_cuda.engine): the generate and chat loops of engine.rs over the
device model (device-side sampling, incremental chat forward on the cached
history) against the same loops over the oracle (oracle forward + the oracle's
Sampler::sample restatement), with the same uniform draws."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

from gguf_cuda import synth
from gguf_cuda.engine import Engine


def encode(text):
    return [(ord(c) * 7919 + 13) % 150000 for c in text]


class OracleModel:
    """The oracle behind the LlamaModel methods the engine calls."""

    def __init__(self, orc, hp, ts):
        self.orc, self.m, self.logits = orc, orc.Model(hp, ts), None
        self.vocab = hp["vocab_size"]

    def forward(self, ids, pos, want_logits=True):
        self.logits = self.m.forward(np.asarray(ids, np.uint32), np.asarray(pos, np.int64))
        return self.logits

    def cache_len(self):
        return self.m.cache_len()

    def reset_cache(self):
        self.m.reset_cache()

    def sample(self, cfg, seen, u):
        return self.orc.sample(self.logits, cfg, seen, u)


@pytest.mark.parametrize("sampler", [dict(temperature=0.0, repeat_penalty=1.3),
                                     dict(temperature=40.0, top_k=40, top_p=0.9, repeat_penalty=1.1)],
                         ids=["greedy-penalty", "sampled"])
def test_chat_two_turns_matches_oracle(ggc, orc, ctx, sampler):
    hp, ts = synth.make_model("qwen2-0.5b-q8_0", n_layers=2, seed=11)
    dev = Engine(ggc.LlamaModel(hp, ts, max_ctx=512, ctx=ctx), encode, eos=None, sampler=sampler, seed=3)
    ref = Engine(OracleModel(orc, hp, ts), encode, eos=None, sampler=sampler, seed=3)
    # turn 1: system + a long user message (> 64 tokens: the batched prefill);
    # turn 2: only the new tokens are forwarded, on top of the cached history
    for text in ("tell me about " + "tensor cores and " * 5, "and the KV cache, briefly, please " * 2):
        a, b = dev.chat(text, 12), ref.chat(text, 12)
        assert a == b
        assert dev.model.cache_len() == ref.model.cache_len()
    dev.reset()
    assert dev.model.cache_len() == 0 and dev.chat_history == []


def test_generate_matches_oracle_and_eos(ggc, orc, ctx):
    hp, ts = synth.make_model("qwen2-0.5b-q8_0", n_layers=2, seed=12)
    s = dict(temperature=40.0, top_k=20, top_p=0.95)
    dev = Engine(ggc.LlamaModel(hp, ts, max_ctx=256, ctx=ctx), encode, sampler=s, seed=5)
    ref = Engine(OracleModel(orc, hp, ts), encode, sampler=s, seed=5)
    prompt = encode("once upon a time")
    a, b = dev.generate(prompt, 16), ref.generate(prompt, 16)
    assert a == b and len(a) == 16
    # EOS ends the loop before the id is emitted
    e = Engine(ggc.LlamaModel(hp, ts, max_ctx=256, ctx=ctx), encode, sampler=s, seed=5, eos=a[3])
    assert e.generate(prompt, 16) == a[:3]


def test_generate_top_k_0_samples_on_the_host(ggc, orc, ctx):
    """top_k = 0 keeps the whole vocabulary (151936 candidates): the engine reads
    the logits back and samples on the host; same ids as the oracle's loop.
    top_p = 1 keeps the candidates in index order, so the pick depends on the
    cumulative sums only (with top_p < 1 the stable sort of ~10^5 nearly equal
    probabilities reorders under the 1e-6 logit differences)."""
    hp, ts = synth.make_model("qwen2-0.5b-q8_0", n_layers=2, seed=13)
    s = dict(temperature=1.0, top_k=0, top_p=1.0, min_p=0.0, repeat_penalty=1.1)
    dev = Engine(ggc.LlamaModel(hp, ts, max_ctx=256, ctx=ctx), encode, sampler=s, seed=7)
    ref = Engine(OracleModel(orc, hp, ts), encode, sampler=s, seed=7)
    assert dev.host_sampling
    prompt = encode("a prompt for the host sampler")
    assert dev.generate(prompt, 12) == ref.generate(prompt, 12)
