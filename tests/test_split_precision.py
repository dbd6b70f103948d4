"""CPU: why the tensor-core expert kernels split every activation into two fp16 terms.

The expert kernels multiply the exact fp16 codes by fp16 activations on the tensor cores. One fp16 term per
value (11 significant bits, scaled per group of 64 by a power of two) leaves the block output about 4e-4 away from
exact arithmetic, far past the 1e-5 rel-L2 parity bar; two terms (hi + lo, 22 bits) leave ~1e-7. So every MMA of
the gate/up and down projections runs on both terms, and the tensor-pipe ceiling for the algorithmic flops of a
compute-bound prefill is half the bf16/fp16 peak. This test measures both on a C1-shape block (dequantised weights
and SwiGLU in float64, the oracle's routing), rounding the activations as the kernels' split does
(expert_tc.cu prep_act_kernel: v * 2^e in [2^14, 2^15) for the group's largest |v|)."""
import numpy as np

import oracle as O

CFG = dict(hidden=2048, E=256, top_k=8, inter=512, sh_inter=512, bits=4)


def _deq(t, e=None):
    w, s, b = t
    if e is not None:
        w, s, b = w[e], s[e], b[e]
    rows = w.shape[0]
    q = ((w[:, :, None] >> (4 * np.arange(8, dtype=np.uint32))) & 15).reshape(rows, -1).astype(np.float64)
    sf = (s.astype(np.uint32) << 16).view(np.float32).astype(np.float64)
    bf = (b.astype(np.uint32) << 16).view(np.float32).astype(np.float64)
    return (q.reshape(rows, -1, 64) * sf[:, :, None] + bf[:, :, None]).reshape(rows, -1)


def _split(v, terms):
    """v rounded as `terms` fp16 terms per group of 64, scaled by the group's power of two."""
    g = v.reshape(-1, 64)
    mx = np.abs(g).max(1, keepdims=True)
    e = 14 - np.floor(np.log2(np.maximum(mx, 1e-300)))
    r, out = g * 2.0 ** e, np.zeros_like(g)
    for _ in range(terms):
        h = r.astype(np.float16).astype(np.float64)
        out += h
        r = r - h
    return (out * 2.0 ** -e).reshape(v.shape)


def test_two_fp16_terms_meet_the_bar_and_one_does_not():
    ob = O.SynthBlock(O.BlockCfg(**CFG), 7)
    a = ob.arrays()
    x = ob.x(4).astype(np.float64)
    _, idx, score = ob.forward(x.astype(np.float32))
    gate_logit = x @ a["sh_gate_f32"].astype(np.float64)

    def block(t, terms):
        xin = _split(x[t], terms) if terms else x[t]

        def mlp(G, U, D):
            g, u = G @ xin, U @ xin
            h = g / (1 + np.exp(-g)) * u
            return D @ (_split(h, terms) if terms else h)
        out = sum(score[t, j] * mlp(_deq(a["gate"], e), _deq(a["up"], e), _deq(a["down"], e))
                  for j, e in enumerate(idx[t]))
        return out + 1 / (1 + np.exp(-gate_logit[t])) * mlp(_deq(a["sh_gate"]), _deq(a["sh_up"]), _deq(a["sh_down"]))

    rel = {terms: max(np.linalg.norm(block(t, terms) - block(t, 0)) / np.linalg.norm(block(t, 0)) for t in range(4))
           for terms in (1, 2)}
    assert rel[1] > 1e-4        # one term: ~4e-4, forty times the parity bar
    assert rel[2] < 1e-6        # two terms: ~1e-7
