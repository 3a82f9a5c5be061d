"""The host restatement of Sampler::sample (gguf_cuda.sampling, used by the
Engine when more than 1024 candidates survive top-k) against the oracle's
restatement of sampler.rs:86-186, on the CPU."""
import numpy as np
import pytest

from gguf_cuda.sampling import device_can_sample, sample_host

CFGS = [dict(temperature=1.0, top_k=0, top_p=0.95, min_p=0.0, repeat_penalty=1.1),
        dict(temperature=0.7, top_k=0, top_p=1.0, min_p=0.0, repeat_penalty=1.0),      # index order kept
        dict(temperature=1.3, top_k=2000, top_p=0.8, min_p=0.05, repeat_penalty=1.2),
        dict(temperature=1.0, top_k=0, top_p=1.0, min_p=0.2, repeat_penalty=1.1),
        dict(temperature=0.0, top_k=0, top_p=0.9, min_p=0.0, repeat_penalty=1.3)]      # greedy


def test_device_limit():
    assert not device_can_sample(dict(temperature=1.0, top_k=0), 32000)
    assert not device_can_sample(dict(temperature=1.0, top_k=1025), 32000)
    assert device_can_sample(dict(temperature=1.0, top_k=40), 151936)
    assert device_can_sample(dict(temperature=0.0, top_k=0), 151936)
    assert device_can_sample(dict(temperature=1.0, top_k=0), 1000)


@pytest.mark.parametrize("ci", range(len(CFGS)))
def test_matches_oracle(orc, ci):
    cfg = CFGS[ci]
    rng = np.random.default_rng(ci)
    logits = (rng.normal(size=4000) * 3).astype(np.float32)
    logits[17] = logits[23] = logits.max()          # a tie at the top
    seen = [17, 5, 3999, 17]
    agree = total = 0
    for u in np.linspace(0.003, 0.997, 120, dtype=np.float32):
        want = orc.sample(logits, cfg, seen, float(u))
        # only draws away from a cumulative boundary decide (exp differs by an ulp between libms)
        if orc.sample(logits, cfg, seen, float(u) - 1e-5) != want or orc.sample(logits, cfg, seen, float(u) + 1e-5) != want:
            continue
        total += 1
        agree += sample_host(logits, cfg, seen, float(u)) == want
    assert total >= 100 and agree == total, (agree, total)
