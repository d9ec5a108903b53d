"""Generate the golden vectors under tests/golden/ (run: python tests/golden/make_golden.py).

The reference (lauritsf/boltz-lumi) ships no golden vectors; its tests pin its
kernels bitwise to reference expressions evaluated with native torch ops.
This script evaluates those same expressions -- with torch's own bf16 tensor
arithmetic on the CPU, no emulation -- on seeded inputs:

* ordered bias softmax: ``s += mask; s += bias; softmax_no_cast(s)`` on bf16
  and fp32 scores with a strided -1e9 mask (tests/test_triangle_softmax.py:14-47);
* SiLU-mul: ``F.silu(a) * b`` on bf16 (tests/test_pair_transition.py:34-51);
* sigmoid gate: ``p * g.sigmoid()`` on bf16 (upstream TriangleMultiplication,
  as kernels/multiplication_gate_hip.cu:16-25 reproduces it);
* gate * fp32 mask promotion: ``(p * g.sigmoid()) * mask[..., None]``
  (multiplication_gate_hip.cu:41-42);
* fp32 diffusion epilogues: ``sigmoid(b) * a + c``, ``sigmoid(a) * b``,
  ``silu(x[:, h:]) * x[:, :h] * c`` (kernels/diffusion_hip.cu:13-27).

The oracle (oracle/numerics.py, oracle/modules.py) re-derives the same values
with explicit fp32 arithmetic and bf16 rounding; tests/test_oracle_golden.py
checks it against these files.
"""

from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent


def softmax_no_cast(t, dim=-1):
    """softmax in the input dtype (upstream primitives.softmax_no_cast)."""
    return torch.nn.functional.softmax(t, dim=dim)


def ordered_softmax_cases():
    g = torch.Generator().manual_seed(46)
    cases = []
    for dtype in (torch.bfloat16, torch.float32):
        for n in (17, 40):
            scores = (torch.randn(1, 3, 4, n, n, generator=g) * 5).to(dtype)
            bias = (torch.randn(1, 1, 4, n, n, generator=g) * 2).to(dtype)
            mask = torch.zeros(1, n, 1, 1, 3).transpose(1, 4)
            mask[:, :, :, :, -3:] = -1e9
            mask[:, 1] = -1e9
            reference = scores.clone()
            reference += mask
            reference += bias
            reference = softmax_no_cast(reference, -1)
            cases.append(dict(scores=scores, bias=bias, mask=mask.contiguous(), expected=reference))
    return cases


def silu_cases():
    g = torch.Generator().manual_seed(81)
    cases = []
    for size in (0, 1, 17, 257, 513, 4096):
        a = (torch.randn(size, generator=g) * 20).bfloat16()
        b = torch.randn(size, generator=g).bfloat16()
        cases.append(dict(a=a, b=b, expected=torch.nn.functional.silu(a) * b))
    return cases


def gate_cases():
    g = torch.Generator().manual_seed(83)
    p = (torch.randn(4096, generator=g) * 3).bfloat16()
    q = (torch.randn(4096, generator=g) * 4).bfloat16()
    pm = (torch.randn(2, 9, 9, 16, generator=g) * 3).bfloat16()
    qm = (torch.randn(2, 9, 9, 16, generator=g) * 4).bfloat16()
    mask = torch.rand(2, 9, 9, generator=g)
    return dict(p=p, g=q, expected=p * q.sigmoid(), pm=pm, gm=qm, mask=mask,
                expected_masked=(pm * qm.sigmoid()) * mask[..., None])


def epilogue_cases():
    g = torch.Generator().manual_seed(85)
    a = torch.randn(37, 768, generator=g) * 3
    b = torch.randn(37, 768, generator=g) * 3
    c = torch.randn(37, 768, generator=g)
    wide = torch.randn(37, 1536, generator=g) * 3
    return dict(a=a, b=b, c=c, wide=wide, modulation=torch.sigmoid(b) * a + c, gate=torch.sigmoid(a) * b,
                swiglu=torch.nn.functional.silu(wide[:, 768:]) * wide[:, :768] * b)


def main():
    torch.save(dict(ordered_softmax=ordered_softmax_cases(), silu=silu_cases(), gate=gate_cases(),
                    epilogue=epilogue_cases()), HERE / "kernel_expressions.pt")
    print("wrote", HERE / "kernel_expressions.pt")


if __name__ == "__main__":
    main()
