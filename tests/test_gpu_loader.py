"""A model loaded from a .gguf file (gguf_cuda.loader) runs exactly as the same
tensors passed directly: bit-identical logits and greedy ids, and within 1e-4 of
the oracle."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

from gguf_cuda import loader, synth


@pytest.mark.parametrize("cfg,n_layers", [("llama2-7b-q4_k_m", 2), ("qwen2-0.5b-q8_0", 2)], ids=["llama2", "qwen2"])
def test_from_gguf_equals_direct(ggc, orc, ctx, tmp_path, cfg, n_layers):
    hp, ts = synth.make_model(cfg, n_layers=n_layers, seed=4)
    p = tmp_path / "model.gguf"
    loader.write_model_gguf(p, hp, ts)
    a = ggc.LlamaModel.from_gguf(p, max_ctx=128, ctx=ctx)
    b = ggc.LlamaModel(hp, ts, max_ctx=128, ctx=ctx)
    prompt = np.random.default_rng(2).integers(0, hp["vocab_size"], size=70).astype(np.uint32)
    pos = np.arange(70, dtype=np.int64)
    la, lb = a.forward(prompt, pos), b.forward(prompt, pos)
    assert np.array_equal(la.view(np.uint32), lb.view(np.uint32))
    lo = orc.Model(hp, ts).forward(prompt, pos)
    assert np.linalg.norm(la.astype(np.float64) - lo) / np.linalg.norm(lo) <= 1e-4
    assert a.decode(8) == b.decode(8)
