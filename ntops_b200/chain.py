"""The Llama-3-8B decoder-layer operator chain used as the end-to-end workload.

It composes only ``ntops_b200.torch`` operators, in the order the benchmark configuration lists
them: rms_norm; q / k / v projections (4096 -> 4096 / 1024 / 1024); rotary position embedding
(head_dim 128, theta 500000, positions 0..S-1, non-interleaved) on q and k; causal GQA
attention (32 query heads, 8 key/value heads); output projection; residual add; rms_norm;
gate / up projections (4096 -> 14336); silu(gate) * up; down projection (14336 -> 4096).

Layouts are chosen so no operator needs a copy: projections produce [B*S, H*D] rows that are
viewed as [B, S, H, D] for RoPE and as [B, H, S, D] (a transposed view) for attention, whose
output keeps the query's memory layout (as the reference's ``torch.empty_like(query)`` does),
so the output projection reads it back as [B*S, H*D] rows.
"""

import torch

import ntops_b200.torch as nt

HIDDEN = 4096
HEADS = 32
KV_HEADS = 8
HEAD_DIM = 128
FFN = 14336
THETA = 500000.0
EPS = 1e-5


class LayerWeights:
    """Random-init bf16 weights ~N(0, 0.02) in [in, out] layout (mm(x, W)); norm weights ones."""

    def __init__(self, device, dtype=torch.bfloat16, seed=0):
        g = torch.Generator(device=device).manual_seed(seed)

        def w(k, n):
            return (torch.randn((k, n), generator=g, device=device, dtype=torch.float32) * 0.02).to(dtype)

        self.wq = w(HIDDEN, HEADS * HEAD_DIM)
        self.wk = w(HIDDEN, KV_HEADS * HEAD_DIM)
        self.wv = w(HIDDEN, KV_HEADS * HEAD_DIM)
        self.wo = w(HEADS * HEAD_DIM, HIDDEN)
        self.wg = w(HIDDEN, FFN)
        self.wu = w(HIDDEN, FFN)
        self.wd = w(FFN, HIDDEN)
        self.norm1 = torch.ones(HIDDEN, device=device, dtype=dtype)
        self.norm2 = torch.ones(HIDDEN, device=device, dtype=dtype)
        from ntops_b200.fused import pack_qkv_weight, pack_swiglu_weight

        self.wgu = pack_swiglu_weight(self.wg, self.wu)  # for the fused SwiGLU projection
        self.wqkv = pack_qkv_weight(self.wq, self.wk, self.wv)  # for the fused QKV + RoPE projection

    def tensors(self):
        return [self.wq, self.wk, self.wv, self.wo, self.wg, self.wu, self.wd, self.norm1, self.norm2]


def rope_tables(seq_len, device, dtype=torch.bfloat16):
    """sin / cos tables [S, D/2] for positions 0..S-1 (same recipe as the reference RoPE test)."""
    inv = THETA ** (-2 * (torch.arange(HEAD_DIM // 2, dtype=torch.float64) / HEAD_DIM))
    pos = torch.arange(seq_len, dtype=torch.float64)[:, None]
    return torch.sin(pos * inv).to(dtype).to(device), torch.cos(pos * inv).to(dtype).to(device)


def gemm_shapes(tokens, fused=True):
    """(M, N, K) of the projection launches of one layer pass, in launch order.  With ``fused``
    the Q / K / V projections are one launch (RoPE in its epilogue) and the gate / up
    projections one launch of width 2 * FFN (SwiGLU in its epilogue)."""
    if fused:
        head = [(tokens, (HEADS + 2 * KV_HEADS) * HEAD_DIM, HIDDEN)]
    else:
        head = [
            (tokens, HEADS * HEAD_DIM, HIDDEN),
            (tokens, KV_HEADS * HEAD_DIM, HIDDEN),
            (tokens, KV_HEADS * HEAD_DIM, HIDDEN),
        ]
    head.append((tokens, HIDDEN, HEADS * HEAD_DIM))
    mlp = [(tokens, 2 * FFN, HIDDEN)] if fused else [(tokens, FFN, HIDDEN), (tokens, FFN, HIDDEN)]
    return head + mlp + [(tokens, HIDDEN, FFN)]


def swiglu_index(fused=True):
    """Position of the fused gate / up (SwiGLU) projection among a pass's GEMM launches."""
    return 2 if fused else None


def layer_flops(batch, seq):
    """Algorithmic FLOPs of one layer pass: 2*M*N*K per projection plus causal attention
    (4 * B * H * S^2 * D scaled by the unmasked fraction (S+1)/(2S))."""
    t = batch * seq
    mm = sum(2 * m * n * k for m, n, k in gemm_shapes(t))
    attn = 4 * batch * HEADS * seq * seq * HEAD_DIM * (seq + 1) / (2 * seq)
    return mm, attn


def layer_forward(x, wts, sin, cos, mm_hook=None, fused=True):
    """One pass of the op chain on x [B, S, 4096] (bf16); returns the down projection [B, S, 4096].

    ``fused`` computes q / k / v and their RoPE as one GEMM with a RoPE epilogue
    (``ntops_b200.fused.qkv_rope_linear``), the residual add and the second rms_norm as one row
    kernel (``ntops_b200.fused.add_rms_norm``) and gate / up / silu / mul as one GEMM with a
    SwiGLU epilogue (``ntops_b200.fused.swiglu_linear``); otherwise each step is its own
    operator.
    ``mm_hook(fn, a, b)``, when given, wraps every projection call (the benchmark times the
    GEMMs with CUDA events through it)."""
    from ntops_b200 import fused as F

    B, S, _ = x.shape
    T = B * S
    mm = nt.mm if mm_hook is None else (lambda a, b: mm_hook(nt.mm, a, b))
    swiglu = F.swiglu_linear if mm_hook is None else (lambda a, b: mm_hook(F.swiglu_linear, a, b))
    x2 = x.view(T, HIDDEN)
    h = nt.rms_norm(x2, (HIDDEN,), wts.norm1, EPS)
    if fused:
        nq, nk = HEADS * HEAD_DIM, KV_HEADS * HEAD_DIM

        def qkv_fn(a, b):
            return F.qkv_rope_linear(a, b, sin, cos, nq + nk)

        qkv = (qkv_fn(h, wts.wqkv) if mm_hook is None else mm_hook(qkv_fn, h, wts.wqkv)).view(B, S, -1)
        q = qkv[..., :nq].view(B, S, HEADS, HEAD_DIM)
        k = qkv[..., nq:nq + nk].view(B, S, KV_HEADS, HEAD_DIM)
        v = qkv[..., nq + nk:].view(B, S, KV_HEADS, HEAD_DIM)
    else:
        q = mm(h, wts.wq).view(B, S, HEADS, HEAD_DIM)
        k = mm(h, wts.wk).view(B, S, KV_HEADS, HEAD_DIM)
        v = mm(h, wts.wv).view(B, S, KV_HEADS, HEAD_DIM)
        q = nt.rotary_position_embedding(q, sin, cos, interleaved=False, inplace=True)
        k = nt.rotary_position_embedding(k, sin, cos, interleaved=False, inplace=True)
    o = nt.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2), is_causal=True,
                                        enable_gqa=True)
    o2 = o.transpose(1, 2).reshape(T, HEADS * HEAD_DIM)  # a view: o keeps q's [B, S, H, D] layout
    attn = mm(o2, wts.wo)
    if fused:
        x2, h2 = F.add_rms_norm(x2, attn, wts.norm2, EPS)
    else:
        x2 = nt.add(x2, attn)
        h2 = nt.rms_norm(x2, (HIDDEN,), wts.norm2, EPS)
    if fused:
        act = swiglu(h2, wts.wgu)
    else:
        gate = mm(h2, wts.wg)
        up = mm(h2, wts.wu)
        act = nt.mul(nt.silu(gate), up)
    down = mm(act, wts.wd)
    return down.view(B, S, HIDDEN)
