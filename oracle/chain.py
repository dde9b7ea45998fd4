"""CPU restatement of the Llama-3-8B layer op chain (test infrastructure and the benchmark's
timed CPU baseline / reference arm only).  Same steps and layouts as ntops_b200/chain.py, built
from the oracle's restatements of the reference operators (oracle/ops.py); ``compute`` selects
float64 (checker) or the input dtype's float32 arithmetic (CPU baseline timing)."""

import torch

from oracle import ops as O

HIDDEN, HEADS, KV_HEADS, HEAD_DIM, FFN, EPS = 4096, 32, 8, 128, 14336, 1e-5
THETA = 500000.0  # RoPE base of Llama-3-8B


def rope_tables(seq_len, dtype=torch.bfloat16):
    """sin / cos tables [S, D/2] for positions 0..S-1 on the CPU (the reference RoPE test's
    recipe, tests/test_rotary_position_embedding.py:32-45, with base THETA)."""
    return O.rope_tables(seq_len, HEAD_DIM, base=THETA, dtype=dtype)


def random_weights(generator, dtype=torch.bfloat16):
    """Random-init weights ~N(0, 0.02) in [in, out] layout on the CPU, in the order
    layer_forward takes them (wq, wk, wv, wo, wg, wu, wd, norm1, norm2); norm weights ones."""

    def w(k, n):
        return (torch.randn((k, n), generator=generator) * 0.02).to(dtype)

    return [w(HIDDEN, HEADS * HEAD_DIM), w(HIDDEN, KV_HEADS * HEAD_DIM), w(HIDDEN, KV_HEADS * HEAD_DIM),
            w(HEADS * HEAD_DIM, HIDDEN), w(HIDDEN, FFN), w(HIDDEN, FFN), w(FFN, HIDDEN),
            torch.ones(HIDDEN, dtype=dtype), torch.ones(HIDDEN, dtype=dtype)]


def layer_forward(x, w, sin, cos):
    """x [B, S, 4096] and the weights (wq, wk, wv, wo, wg, wu, wd, norm1, norm2) on the CPU."""
    wq, wk, wv, wo, wg, wu, wd, n1, n2 = w
    B, S, _ = x.shape
    T = B * S
    x2 = x.reshape(T, HIDDEN)
    h = O.rms_norm(x2, (HIDDEN,), n1, EPS)
    q = O.mm(h, wq).view(B, S, HEADS, HEAD_DIM)
    k = O.mm(h, wk).view(B, S, KV_HEADS, HEAD_DIM)
    v = O.mm(h, wv).view(B, S, KV_HEADS, HEAD_DIM)
    q = O.rotary_position_embedding(q, sin, cos, interleaved=False)
    k = O.rotary_position_embedding(k, sin, cos, interleaved=False)
    o = O.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2), None, True,
                                       block=256)
    o2 = o.transpose(1, 2).reshape(T, HEADS * HEAD_DIM)
    x2 = O.add(x2, O.mm(o2, wo))
    h2 = O.rms_norm(x2, (HIDDEN,), n2, EPS)
    act = O.mul(O.silu(O.mm(h2, wg)), O.mm(h2, wu))
    return O.mm(act, wd).view(B, S, HIDDEN)


def layer_forward_torch_cpu(x, w, sin, cos):
    """The same chain on PyTorch's own CPU operators in the workload dtype (bf16) — the CPU
    implementation the benchmark reports as its baseline."""
    import torch.nn.functional as F

    wq, wk, wv, wo, wg, wu, wd, n1, n2 = w
    B, S, _ = x.shape
    T = B * S
    x2 = x.reshape(T, HIDDEN)
    h = F.rms_norm(x2, (HIDDEN,), n1, EPS)
    q = (h @ wq).view(B, S, HEADS, HEAD_DIM)
    k = (h @ wk).view(B, S, KV_HEADS, HEAD_DIM)
    v = (h @ wv).view(B, S, KV_HEADS, HEAD_DIM)

    def rope(t):
        half = HEAD_DIM // 2
        t0, t1 = t[..., :half], t[..., half:]
        s4, c4 = sin[None, :, None, :], cos[None, :, None, :]
        return torch.cat((t0 * c4 - t1 * s4, t0 * s4 + t1 * c4), -1)

    q, k = rope(q), rope(k)
    o = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2), is_causal=True,
                                       enable_gqa=True)
    o2 = o.transpose(1, 2).reshape(T, HEADS * HEAD_DIM)
    x2 = x2 + o2 @ wo
    h2 = F.rms_norm(x2, (HIDDEN,), n2, EPS)
    act = F.silu(h2 @ wg) * (h2 @ wu)
    return (act @ wd).view(B, S, HIDDEN)
