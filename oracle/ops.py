"""Float64 CPU restatements of the reference operators (test infrastructure only).

Every function takes and returns CPU torch tensors.  Arithmetic runs in float64 and the result
is rounded once to the output dtype, except integer / bool operators, which run in their own
integer type (bit-exact).  Each function cites the reference lines (paths inside the ntops
project) whose algorithm it restates.  Broadcasting and type promotion follow torch, which is
what the reference's tests compare against.
"""

import math

import torch

F64 = torch.float64


def _f(t):
    return t.to(F64)


def _promote(a, b):
    if not isinstance(a, torch.Tensor):
        a = torch.tensor(a, dtype=torch.result_type(b, a))
    if not isinstance(b, torch.Tensor):
        b = torch.tensor(b, dtype=torch.result_type(a, b))
    dt = torch.result_type(a, b)
    shape = torch.broadcast_shapes(a.shape, b.shape)
    return a.to(dt).expand(shape), b.to(dt).expand(shape), dt


# ----------------------------------------------------------------------- elementwise ------
def add(input, other, alpha=1):
    """kernels/add.py:9-10: input + alpha * other."""
    a, b, dt = _promote(input, other)
    if dt.is_floating_point:
        return (_f(a) + alpha * _f(b)).to(dt)
    if dt == torch.bool:
        return a | (b & bool(alpha))
    return (a + int(alpha) * b).to(dt)


def sub(input, other, alpha=1):
    """kernels/sub.py:9-10: input - alpha * other."""
    a, b, dt = _promote(input, other)
    if dt.is_floating_point:
        return (_f(a) - alpha * _f(b)).to(dt)
    return (a - int(alpha) * b).to(dt)


def mul(input, other):
    """kernels/mul.py:8-9."""
    a, b, dt = _promote(input, other)
    if dt.is_floating_point:
        return (_f(a) * _f(b)).to(dt)
    return a * b


def _floor_divide_float(a, b):
    """Floor division of floating-point a / b in a's dtype, the algorithm of CPython's
    float_divmod (Objects/floatobject.c), which torch's div(rounding_mode="floor") follows:
    remainder by fmod, quotient (a - mod) / b moved down by one when the remainder's sign differs
    from the divisor's, then rounded to the nearest integer from below; b = 0 gives a / b."""
    mod = torch.fmod(a, b)
    div = (a - mod) / b
    div = torch.where((mod != 0) & ((b < 0) != (mod < 0)), div - 1, div)
    fd = torch.floor(div)
    fd = torch.where(div - fd > 0.5, fd + 1, fd)
    fd = torch.where(div == 0, torch.copysign(torch.zeros_like(div), a / b), fd)
    return torch.where(b == 0, a / b, fd)


def div(input, other, rounding_mode=None):
    """kernels/div.py:9-18: true, trunc (cast of the quotient to int64) or floor division.

    True division runs in float64, rounded once.  The rounding modes give integer-valued
    results that a float64 quotient could place on the other side of an integer, so they restate
    the exact arithmetic instead: the quotient in the compute dtype (float32 for 16-bit and
    float32 inputs, float64 for float64), then trunc, or the floor-division algorithm above;
    the integer-valued result is rounded once to the input dtype."""
    a, b, dt = _promote(input, other)
    if rounding_mode is None:
        out_dt = dt if dt.is_floating_point else torch.get_default_dtype()
        return (_f(a) / _f(b)).to(out_dt)
    if dt.is_floating_point:
        ct = F64 if dt == F64 else torch.float32
        ac, bc = a.to(ct), b.to(ct)
        q = torch.trunc(ac / bc) if rounding_mode == "trunc" else _floor_divide_float(ac, bc)
        return q.to(dt)
    if rounding_mode == "trunc":
        return torch.div(a, b, rounding_mode="trunc")
    return torch.div(a, b, rounding_mode="floor")


def pow(input, exponent):
    """kernels/pow.py:9-10 (libdevice.pow): x ** e, NaN for negative x with a fractional e."""
    a, b, dt = _promote(input, exponent)
    if dt.is_floating_point:
        return torch.pow(_f(a), _f(b)).to(dt)
    return torch.pow(a, b)


def _compare(fn, input, other):
    a, b, dt = _promote(input, other)
    if dt.is_floating_point:
        return fn(_f(a), _f(b))
    return fn(a, b)


def eq(input, other):
    """kernels/eq.py:8-9 (bool result, as torch)."""
    return _compare(torch.eq, input, other)


def ne(input, other):
    """kernels/ne.py:8-9."""
    return _compare(torch.ne, input, other)


def lt(input, other):
    """kernels/lt.py:8-9."""
    return _compare(torch.lt, input, other)


def le(input, other):
    """kernels/le.py:8-9."""
    return _compare(torch.le, input, other)


def gt(input, other):
    """kernels/gt.py:8-9."""
    return _compare(torch.gt, input, other)


def ge(input, other):
    """kernels/ge.py:8-9."""
    return _compare(torch.ge, input, other)


def bitwise_and(input, other):
    """kernels/bitwise_and.py:8-9."""
    a, b, _ = _promote(input, other)
    return a & b


def bitwise_or(input, other):
    """kernels/bitwise_or.py:8-9."""
    a, b, _ = _promote(input, other)
    return a | b


def bitwise_not(input):
    """kernels/bitwise_not.py:9-14: ~x, logical not for bool."""
    if input.dtype == torch.bool:
        return torch.logical_not(input)
    return ~input


def _unary_float(fn, input):
    x = input if input.is_floating_point() else input.to(torch.get_default_dtype())
    return fn(_f(x)).to(x.dtype)


def neg(input):
    """kernels/neg.py:8."""
    return _unary_float(torch.neg, input) if input.is_floating_point() else -input


def abs(input):
    """kernels/abs.py:9-10."""
    return _unary_float(torch.abs, input) if input.is_floating_point() else torch.abs(input)


def relu(input):
    """kernels/relu.py:8-9: max(0, x) (NaN propagates, as torch)."""
    if not input.is_floating_point():
        return torch.clamp_min(input, 0)
    return _unary_float(torch.relu, input)


def exp(input):
    """kernels/exp.py:9-10."""
    return _unary_float(torch.exp, input)


def sigmoid(input):
    """kernels/sigmoid.py:9-10: 1 / (1 + exp(-x))."""
    return _unary_float(lambda x: 1.0 / (1.0 + torch.exp(-x)), input)


def silu(input):
    """kernels/silu.py:9-10: x / (1 + exp(-x)) with exp in float."""
    return _unary_float(lambda x: x / (1.0 + torch.exp(-x)), input)


def gelu(input, approximate="none"):
    """kernels/gelu.py:10-26: erf form, or tanh form with sqrt(2/pi) (x + 0.044715 x^3)."""
    if approximate == "tanh":
        fn = lambda x: 0.5 * x * (1 + torch.tanh(math.sqrt(2 / math.pi) * (x + 0.044715 * x**3)))  # noqa: E731
    else:
        fn = lambda x: x * 0.5 * (1 + torch.erf(x / math.sqrt(2.0)))  # noqa: E731
    return _unary_float(fn, input)


def tanh(input):
    """kernels/tanh.py:9-12 (exp formula; computed here with tanh, equal where the formula is finite)."""
    return _unary_float(torch.tanh, input)


def rsqrt(input):
    """kernels/rsqrt.py:9-10: rsqrt in fp32."""
    return _unary_float(lambda x: 1.0 / torch.sqrt(x), input)


def sin(input):
    """kernels/sin.py:9."""
    return _unary_float(torch.sin, input)


def cos(input):
    """kernels/cos.py:9."""
    return _unary_float(torch.cos, input)


def isnan(input):
    """kernels/isnan.py:8: x != x (bool result, as torch)."""
    return input != input


def isinf(input):
    """kernels/isinf.py:8-11: x == +inf or x == -inf (bool result)."""
    if not input.is_floating_point():
        return torch.zeros(input.shape, dtype=torch.bool)
    return (input == float("inf")) | (input == float("-inf"))


def clamp(input, min=None, max=None):
    """kernels/clamp.py:9-10: min(max(x, lo), hi) (NaN propagates; lo applied first)."""
    if input.is_floating_point():
        x = _f(input)
        lo = _f(min) if isinstance(min, torch.Tensor) else min
        hi = _f(max) if isinstance(max, torch.Tensor) else max
        return torch.clamp(x, lo, hi).to(input.dtype)
    return torch.clamp(input, min, max)


# --------------------------------------------------------------------- row reductions -----
def rms_norm(input, normalized_shape, weight=None, eps=None):
    """kernels/rms_norm.py:10-20 with torch/rms_norm.py:15-21 defaults:
    rms = sqrt(sum(x^2) / n + eps); y = x / rms * w; eps defaults to finfo(dtype).eps."""
    if isinstance(normalized_shape, int):
        normalized_shape = (normalized_shape,)
    if eps is None:
        eps = torch.finfo(input.dtype).eps
    dims = tuple(range(-len(normalized_shape), 0))
    n = math.prod(normalized_shape)
    x = _f(input)
    rms = torch.sqrt((x * x).sum(dims, keepdim=True) / n + eps)
    y = x / rms
    if weight is not None:
        y = y * _f(weight)
    return y.to(input.dtype)


def layer_norm(input, normalized_shape, weight=None, bias=None, eps=1e-5):
    """kernels/layer_norm.py:11-31: mean, biased variance of (x - mean), (x - mean) / sqrt(var + eps)
    * w + b."""
    if isinstance(normalized_shape, int):
        normalized_shape = (normalized_shape,)
    dims = tuple(range(-len(normalized_shape), 0))
    n = math.prod(normalized_shape)
    x = _f(input)
    mean = x.sum(dims, keepdim=True) / n
    var = ((x - mean) ** 2).sum(dims, keepdim=True) / n
    y = (x - mean) / torch.sqrt(var + eps)
    if weight is not None:
        y = y * _f(weight)
    if bias is not None:
        y = y + _f(bias)
    return y.to(input.dtype)


def softmax(input, dim, dtype=None, block=64):
    """kernels/softmax.py:14-29: pass 1 walks the row in blocks keeping a running max and a
    denominator rescaled by exp(prev_max - curr_max); pass 2 writes exp(x - max) / denominator."""
    out_dtype = dtype if dtype is not None else input.dtype
    x = _f(input).movedim(dim, -1)
    n = x.shape[-1]
    prev_max = torch.full(x.shape[:-1], float("-inf"), dtype=F64)
    den = torch.zeros(x.shape[:-1], dtype=F64)
    for s in range(0, n, block):
        xb = x[..., s : s + block]
        curr = torch.maximum(prev_max, xb.max(-1).values)
        safe = torch.where(torch.isinf(curr) & (curr < 0), torch.zeros_like(curr), curr)
        den = den * torch.exp(prev_max - safe) + torch.exp(xb - safe[..., None]).sum(-1)
        prev_max = curr
    y = torch.exp(x - prev_max[..., None]) / den[..., None]
    return y.movedim(-1, dim).to(out_dtype)


# ------------------------------------------------------------------------------ RoPE ------
def rotary_position_embedding(input, sin_table, cos_table, interleaved=True):
    """kernels/rotary_position_embedding.py:6-47: pairs (2i, 2i+1) when interleaved, else
    (i, i + D/2); (x0, x1) -> (x0 cos - x1 sin, x0 sin + x1 cos) with tables [S, D/2] broadcast
    over batch and heads (torch/rotary_position_embedding.py:17-18)."""
    x = _f(input)
    s = _f(sin_table)[None, :, None, :]
    c = _f(cos_table)[None, :, None, :]
    d = x.shape[-1]
    if interleaved:
        x0, x1 = x[..., 0::2], x[..., 1::2]
    else:
        x0, x1 = x[..., : d // 2], x[..., d // 2 :]
    y0 = x0 * c - x1 * s
    y1 = x0 * s + x1 * c
    y = torch.empty_like(x)
    if interleaved:
        y[..., 0::2], y[..., 1::2] = y0, y1
    else:
        y[..., : d // 2], y[..., d // 2 :] = y0, y1
    return y.to(input.dtype)


def rope_tables(seq_len, emb_dim, base=10000.0, dtype=torch.float32):
    """Table recipe of the reference's RoPE test (tests/test_rotary_position_embedding.py:32-45):
    theta_i = base^(-2i/D), sin/cos(position * theta) for positions 0..S-1."""
    theta = base ** (-2 * (torch.arange(emb_dim // 2, dtype=torch.float64) / emb_dim))
    pos = torch.arange(seq_len, dtype=torch.float64).unsqueeze(1)
    return torch.sin(pos * theta).to(dtype), torch.cos(pos * theta).to(dtype)


# ------------------------------------------------------------------------------ GEMM ------
def mm(input, mat2):
    """kernels/mm.py:54-65: K loop of dot products into a wide accumulator; output in input dtype."""
    return (_f(input) @ _f(mat2)).to(input.dtype)


def bmm(input, mat2):
    """kernels/bmm.py (same application as mm over the batch)."""
    return (_f(input) @ _f(mat2)).to(input.dtype)


def addmm(input, mat1, mat2, beta=1, alpha=1):
    """kernels/addmm.py:64-67: beta * input + alpha * (mat1 @ mat2); output in input's dtype."""
    return (beta * _f(input) + alpha * (_f(mat1) @ _f(mat2))).to(input.dtype)


def matmul(input, other):
    """torch/matmul.py:9-18: 2-D -> mm, otherwise bmm of the 3-D forms."""
    return (_f(input) @ _f(other)).to(input.dtype)


# ------------------------------------------------------------------------- attention ------
def scaled_dot_product_attention(query, key, value, attn_mask=None, is_causal=False, scale=None,
                                 causal_variant=1, block=64):
    """kernels/scaled_dot_product_attention.py:154-201: per q-head, loop over KV blocks:
    S = Q K^T (query prescaled by scale * log2(e), :166), out-of-range keys masked, additive mask,
    causal mask (upper-left k <= q, :188; lower-right k <= q + Skv - Sq, :180-186), online softmax
    in base 2 (:192-198), O / l (:200).  GQA maps q-head h to kv-head h // (Hq / Hkv) (:38-45).
    The additive mask is taken in natural-log units (multiplied by log2(e) in the base-2 domain),
    which is torch's semantics and equals the reference on the 0 / -inf masks its tests use."""
    log2e = 1.4426950408889634
    q, k, v = _f(query), _f(key), _f(value)
    B, Hq, Sq, D = q.shape
    Hkv, Skv = k.shape[1], k.shape[2]
    if scale is None:
        scale = 1 / math.sqrt(D)
    g = Hq // Hkv
    k = k.repeat_interleave(g, dim=1)
    v = v.repeat_interleave(g, dim=1)
    mask = None
    if attn_mask is not None:
        if attn_mask.dtype == torch.bool:
            mask = torch.where(attn_mask, 0.0, float("-inf")).to(F64)
        else:
            mask = _f(attn_mask)
        mask = mask.expand(B, Hq, Sq, Skv)
    qi = torch.arange(Sq)[:, None]
    off = (Skv - Sq) if causal_variant == 2 else 0
    acc = torch.zeros(B, Hq, Sq, v.shape[-1], dtype=F64)
    lse = torch.zeros(B, Hq, Sq, dtype=F64)
    mx = torch.full((B, Hq, Sq), float("-inf"), dtype=F64)
    qs = q * (scale * log2e)
    for s in range(0, Skv, block):
        kb, vb = k[:, :, s : s + block], v[:, :, s : s + block]
        qk = qs @ kb.transpose(-1, -2)
        kj = torch.arange(s, s + kb.shape[2])[None, :]
        if mask is not None:
            qk = qk + mask[..., s : s + block] * log2e
        if is_causal:
            qk = torch.where(qi + off >= kj, qk, torch.tensor(float("-inf"), dtype=F64))
        nxt = torch.maximum(mx, qk.max(-1).values)
        safe = torch.where(torch.isinf(nxt) & (nxt < 0), torch.zeros_like(nxt), nxt)
        p = torch.exp2(qk - safe[..., None])
        alpha = torch.exp2(mx - safe)
        acc = acc * alpha[..., None] + p @ vb
        lse = lse * alpha + p.sum(-1)
        mx = nxt
    return (acc / lse[..., None]).to(value.dtype)


# --------------------------------------------------------- special elementwise (§ f2) -----
def copysign(input, other):
    """kernels/copysign.py:13-53: magnitude bits of input with the sign bit of other."""
    a, b, dt = _promote(input, other)
    out_dt = dt if dt.is_floating_point else torch.get_default_dtype()
    return torch.copysign(_f(a), _f(b)).to(out_dt)


def nextafter(input, other):
    """kernels/nextafter.py:13-123: one step of the IEEE encoding from input toward other
    (other itself when equal, NaN when either is NaN, the smallest subnormal from zero)."""
    a, b, dt = _promote(input, other)
    if dt in (torch.float32, torch.float64):
        return torch.nextafter(a, b)
    ia = a.contiguous().view(torch.int16).to(torch.int32) & 0xFFFF
    ib = b.contiguous().view(torch.int16).to(torch.int32) & 0xFFFF
    fa, fb = a.double(), b.double()
    step_up = ia + 1
    step_dn = ia - 1
    away = (fa < fb) == ((ia & 0x8000) == 0)
    r = torch.where(away, step_up, step_dn)
    r = torch.where((ia & 0x7FFF) == 0, (ib & 0x8000) | 1, r)
    r = torch.where(fa == fb, ib, r)
    out = (r & 0xFFFF).to(torch.int32)
    out = torch.where(out >= 0x8000, out - 0x10000, out).to(torch.int16).view(dt)
    nan = torch.isnan(fa) | torch.isnan(fb)
    return torch.where(nan, torch.tensor(float("nan"), dtype=dt), out)


def lcm(input, other):
    """kernels/lcm.py:14-128: |a / gcd(a, b) * b|, 0 when either is 0."""
    a, b, _ = _promote(input, other)
    return torch.lcm(a, b)


def rad2deg(input):
    """kernels/rad2deg.py:13-19: x * 180 / pi."""
    return _unary_float(lambda x: x * (180.0 / math.pi), input)


def frac(input):
    """kernels/frac.py:12-27: x - trunc(x)."""
    return _unary_float(lambda x: x - torch.trunc(x), input)


def lgamma(input):
    """kernels/lgamma.py:14-29: log |gamma(x)|."""
    return _unary_float(torch.lgamma, input)


# ------------------------------------------------------------------------ dropout ---------
def philox_rand(seed, offsets):
    """The uniform the reference's dropout draws per element (kernels/dropout.py:10, `ntl.rand`):
    Triton 3.6's tl.rand (third-party, triton/language/random.py `randint4x` / `philox_impl` /
    `uint_to_uniform_float`), restated from the published Philox-4x32-10 algorithm (Salmon et
    al., SC 2011): counter (offset low word, offset high word, 0, 0), key (seed low word, seed
    high word), 10 rounds with multipliers 0xD2511F53 / 0xCD9E8D57 and key increments 0x9E3779B9 /
    0xBB67AE85; the first output word x (as int32) maps to (x < 0 ? -x - 1 : x) * 4.6566127342e-10
    in fp32.  numpy, uint64 arithmetic masked to 32 bits."""
    import numpy as np

    m = np.uint64(0xFFFFFFFF)
    off = np.asarray(offsets, dtype=np.int64).astype(np.uint64)
    c0, c1 = off & m, (off >> np.uint64(32)) & m
    c2 = np.zeros_like(c0)
    c3 = np.zeros_like(c0)
    k0, k1 = np.uint64(seed & 0xFFFFFFFF), np.uint64((seed >> 32) & 0xFFFFFFFF)
    ra, rb = np.uint64(0xD2511F53), np.uint64(0xCD9E8D57)
    for _ in range(10):
        pb, pa = rb * c2, ra * c0
        c0, c2 = ((pb >> np.uint64(32)) ^ c1 ^ k0) & m, ((pa >> np.uint64(32)) ^ c3 ^ k1) & m
        c1, c3 = pb & m, pa & m
        k0, k1 = (k0 + np.uint64(0x9E3779B9)) & m, (k1 + np.uint64(0xBB67AE85)) & m
    x = c0.astype(np.uint32).view(np.int32).astype(np.int64)
    x = np.where(x < 0, -x - 1, x)
    return torch.from_numpy((x.astype(np.float32) * np.float32(4.6566127342e-10)).astype(np.float32))


def round_once(t64, dtype):
    """float64 -> dtype with ONE round-to-nearest-even.  torch's float64 -> float16 / bfloat16
    conversion on the CPU goes through float32 (two roundings, which differ near midpoints); an
    intermediate float32 rounded to odd (truncate, then set the last bit when inexact) keeps the
    second rounding exact, the standard fix for double rounding."""
    if dtype not in (torch.float16, torch.bfloat16):
        return t64.to(dtype)
    r = t64.to(torch.float32)
    back = r.to(F64)
    over = back.abs() > t64.abs()
    trunc = torch.where(over, torch.nextafter(r, torch.zeros_like(r)), r)
    inexact = trunc.to(F64) != t64
    bits = trunc.view(torch.int32)
    odd = torch.where(inexact & torch.isfinite(trunc), bits | 1, bits).view(torch.float32)
    return odd.to(dtype)


def dropout(input, p, seed):
    """kernels/dropout.py:10-11: where(rand(seed, offset) > p, input / (1 - p), 0) with the
    element's row-major index as offset; compare and divide in fp64 (p is an fp64 scalar there),
    one rounding to the output dtype."""
    r = philox_rand(seed, range(input.numel())).reshape(input.shape).double()
    y = torch.where(r > p, _f(input) / (1.0 - p), torch.zeros((), dtype=F64))
    return round_once(y, input.dtype)


# -------------------------------------------------------------------------- conv2d --------
def conv2d(input, weight, bias=None, stride=1, padding=0, dilation=1):
    """kernels/conv2d.py:16-115 (padded input tiled into (C, R, S) patches, mm with the weight
    flattened to [K, C*R*S], bias in the epilogue; NCHW): computed here in float64 with
    torch's CPU convolution, the oracle of the reference's tests/test_conv2d.py."""
    import torch.nn.functional as Fn

    y = Fn.conv2d(_f(input), _f(weight), None if bias is None else _f(bias), stride=stride, padding=padding,
                  dilation=dilation)
    return y.to(input.dtype)
