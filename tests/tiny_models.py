"""The two tiny F32 llama models of the reference's tests, as role-ordered tensors.

* forward_runs: src/infer/model/llama.rs:789-899 (1 layer, d=4, 2 heads, 1 kv head,
  ffn 6, vocab 8; all weights zero except token_embd row 1 = 1.0).
* min_llama: tests/inference.rs:80-214 (2 layers, same dims; norms 1.0; ffn.w1,
  ffn.w3 and output hold 0.5 at every fourth float, all else zero).
Role order: token_embd, output_norm, output, then per layer attn_norm, attn_q,
attn_q.bias, attn_k, attn_k.bias, attn_v, attn_v.bias, attn_output, ffn_norm,
ffn_up (= ffn.w1), ffn_gate (= ffn.w2), ffn_down (= ffn.w3).
"""
import numpy as np

F32 = 0
D, Q, KV, F, VOCAB = 4, 2, 1, 6, 8
HD = D // Q


def _t(values):
    v = np.ascontiguousarray(values, dtype=np.float32)
    return {"raw": v.view(np.uint8), "dtype": F32, "n_elements": v.size}


def forward_runs_hp():
    return dict(vocab_size=VOCAB, embed_dim=D, n_heads=Q, n_kv_heads=KV, ffn_dim=F, n_layers=1, rope_freq_base=10000.0)


def forward_runs_tensors():
    embd = np.zeros(D * VOCAB, np.float32)
    embd[D:2 * D] = 1.0
    z = lambda n: _t(np.zeros(n, np.float32))
    return [_t(embd), z(D), z(D * VOCAB),
            z(D), z(Q * HD * D), None, z(KV * HD * D), None, z(KV * HD * D), None, z(D * Q * HD),
            z(D), z(F * D), z(F * D), z(D * F)]


def min_llama_hp():
    return dict(vocab_size=VOCAB, embed_dim=D, n_heads=Q, n_kv_heads=KV, ffn_dim=F, n_layers=2, rope_freq_base=10000.0)


def min_llama_tensors():
    def sparse(n):
        v = np.zeros(n, np.float32)
        v[::4] = 0.5
        return _t(v)
    z = lambda n: _t(np.zeros(n, np.float32))
    one = lambda n: _t(np.ones(n, np.float32))
    ts = [z(VOCAB * D), one(D), sparse(VOCAB * D)]
    for _ in range(2):
        ts += [one(D), z(Q * HD * D), None, z(KV * HD * D), None, z(KV * HD * D), None, z(D * Q * HD),
               one(D), sparse(F * D), z(F * D), sparse(D * F)]
    return ts
