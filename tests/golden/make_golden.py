"""Generates tests/golden/golden.pt: small seeded inputs and the outputs PyTorch's CPU operators
give for them in float64 — the oracle the reference's own tests compare ntops against
(tests/test_<op>.py in the ntops project).  Run from the repository root:

    python tests/golden/make_golden.py

The fixtures pin the CPU oracle (tests/test_oracle.py) and the CUDA path
(tests/test_golden_gpu.py) to the same committed numbers.
"""

import math
import os

import torch
import torch.nn.functional as F

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden.pt")


def main():
    g = torch.Generator().manual_seed(0)

    def rn(*shape, dtype=torch.float32, scale=1.0):
        return (torch.randn(shape, generator=g, dtype=torch.float64) * scale).to(dtype)

    cases = []

    def add(name, fn, inputs, kwargs=None):
        kwargs = kwargs or {}
        d64 = [t.double() if isinstance(t, torch.Tensor) and t.is_floating_point() else t for t in inputs]
        out = fn(*d64, **kwargs)
        out_dtype = inputs[0].dtype if inputs[0].is_floating_point() else out.dtype
        if isinstance(out, torch.Tensor) and out.is_floating_point():
            out = out.to(out_dtype)
        cases.append({"op": name, "inputs": inputs, "kwargs": kwargs, "expected": out})

    for dt in (torch.float32, torch.float16, torch.bfloat16):
        x, y = rn(7, 33, dtype=dt), rn(7, 33, dtype=dt)
        add("add", lambda a, b, alpha: torch.add(a, b, alpha=alpha), [x, y, 0.5])
        add("mul", torch.mul, [x, y])
        add("div", torch.div, [x, y])
        add("silu", F.silu, [x])
        add("gelu_tanh", lambda a: F.gelu(a, approximate="tanh"), [x])
        add("gelu", F.gelu, [x])
        add("sigmoid", torch.sigmoid, [x])
        add("exp", torch.exp, [x])
        add("clamp", lambda a: torch.clamp(a, -1, 1), [x])
        add("pow", torch.pow, [(torch.rand(7, 33, generator=g) * 8 - 4).to(dt),
                               (torch.rand(7, 33, generator=g) * 1.5 + 0.5).to(dt)])
        add("rms_norm", lambda a, w: F.rms_norm(a, (33,), w, 1e-6), [x, rn(33, dtype=dt)])
        add("layer_norm", lambda a, w, b: F.layer_norm(a, (33,), w, b, 1e-5), [x, rn(33, dtype=dt), rn(33, dtype=dt)])
        add("softmax", lambda a: torch.softmax(a, -1), [rn(5, 100, dtype=dt, scale=2.0)])
    xi, yi = (torch.randint(-2**31, 2**31 - 1, (1000,), generator=g, dtype=torch.int64).to(torch.int32) for _ in range(2))
    cases.append({"op": "bitwise_and", "inputs": [xi, yi], "kwargs": {}, "expected": xi & yi})
    cases.append({"op": "bitwise_or", "inputs": [xi, yi], "kwargs": {}, "expected": xi | yi})
    cases.append({"op": "bitwise_not", "inputs": [xi], "kwargs": {}, "expected": ~xi})
    xh, yh = rn(1000, dtype=torch.float16), rn(1000, dtype=torch.float16)
    yh[::4] = xh[::4]
    cases.append({"op": "eq", "inputs": [xh, yh], "kwargs": {}, "expected": xh == yh})
    cases.append({"op": "lt", "inputs": [xh, yh], "kwargs": {}, "expected": xh < yh})

    # RoPE: the reference test's torch restatement (tests/test_rotary_position_embedding.py:8-29)
    B, S, H, D = 2, 16, 3, 64
    xr = rn(B, S, H, D)
    theta = 500000.0 ** (-2 * (torch.arange(D // 2, dtype=torch.float64) / D))
    pos = torch.arange(S, dtype=torch.float64)[:, None]
    sn, cs = torch.sin(pos * theta), torch.cos(pos * theta)
    for inter in (False, True):
        x64 = xr.double()
        if inter:
            x0, x1 = x64[..., 0::2], x64[..., 1::2]
        else:
            x0, x1 = x64[..., : D // 2], x64[..., D // 2 :]
        s4, c4 = sn[None, :, None, :], cs[None, :, None, :]
        y0, y1 = x0 * c4 - x1 * s4, x0 * s4 + x1 * c4
        y = torch.stack((y0, y1), -1).reshape(B, S, H, D) if inter else torch.cat((y0, y1), -1)
        cases.append({"op": "rope", "inputs": [xr, sn.float(), cs.float()], "kwargs": {"interleaved": inter},
                      "expected": y.float()})

    # GEMM
    for dt in (torch.float32, torch.bfloat16):
        a, b, c = rn(40, 72, dtype=dt), rn(72, 24, dtype=dt), rn(40, 24, dtype=dt)
        add("mm", torch.mm, [a, b])
        add("addmm", lambda i, x, y: torch.addmm(i, x, y, beta=0.5, alpha=2.0), [c, a, b])
        add("bmm", torch.bmm, [rn(2, 40, 72, dtype=dt), rn(2, 72, 24, dtype=dt)])

    # Attention (GQA 4 -> 2 heads), causal and not, bf16 and fp32
    for dt in (torch.float32, torch.bfloat16):
        q, k, v = rn(1, 4, 48, 64, dtype=dt), rn(1, 2, 80, 64, dtype=dt), rn(1, 2, 80, 64, dtype=dt)
        add("sdpa", lambda q_, k_, v_: F.scaled_dot_product_attention(q_, k_, v_, enable_gqa=True), [q, k, v])
        qc = rn(1, 4, 80, 64, dtype=dt)
        add("sdpa_causal", lambda q_, k_, v_: F.scaled_dot_product_attention(q_, k_, v_, is_causal=True, enable_gqa=True),
            [qc, k, v])

    torch.save(cases, OUT)
    print(f"wrote {len(cases)} cases to {OUT} ({os.path.getsize(OUT)} bytes)")


if __name__ == "__main__":
    main()
