"""Run one pair-path op (or a whole Pairformer block) a few times, for profilers.

    python -m boltz_lumi_b200.profile_ops --op att_start --n 512 --iters 3

Ops: tri_mul_out, tri_mul_in, att_start, att_end, transition, block.  Inputs
and weights are the benchmark's synthetic ones (seeded); z is updated in
place like in the Pairformer block.  Prints the mean device time per call.
"""

import argparse

import torch

from . import forwards, layers


def seeded_block(seed=1234):
    module = layers.PairformerLayer()
    g = torch.Generator().manual_seed(seed)
    with torch.no_grad():
        for name, p in module.named_parameters():
            mean = 1.0 if "norm" in name and name.endswith("weight") else 0.0
            p.copy_(torch.randn(p.shape, generator=g) * (1.0 / 128) ** 0.5 + mean)
    return module.eval()


def main():
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("--op", default="block",
                        choices=["tri_mul_out", "tri_mul_in", "att_start", "att_end", "transition", "block"])
    parser.add_argument("--n", type=int, default=512)
    parser.add_argument("--iters", type=int, default=3)
    args = parser.parse_args()
    block = seeded_block().cuda()
    g = torch.Generator().manual_seed(7)
    n = args.n
    z = torch.randn(1, n, n, 128, generator=g).cuda()
    s = torch.randn(1, n, 384, generator=g).cuda()
    mask = torch.ones(1, n, device="cuda")
    pmask = torch.ones(1, n, n, device="cuda")
    ops = {
        "tri_mul_out": lambda: forwards.triangle_multiplication_forward(block.tri_mul_out, z, pmask, residual=z),
        "tri_mul_in": lambda: forwards.triangle_multiplication_forward(block.tri_mul_in, z, pmask, residual=z),
        "att_start": lambda: forwards.triangle_attention_forward(block.tri_att_start, z, pmask, residual=z),
        "att_end": lambda: forwards.triangle_attention_forward(block.tri_att_end, z, pmask, residual=z),
        "transition": lambda: forwards.transition_forward(block.transition_z, z, residual=z),
        "block": lambda: block(s, z, mask, pmask),
    }
    fn = ops[args.op]
    with torch.inference_mode():
        fn()
        torch.cuda.synchronize()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(args.iters):
            fn()
        end.record()
        torch.cuda.synchronize()
    print(f"{args.op} n={n}: {start.elapsed_time(end) / args.iters:.4f} ms per call")


if __name__ == "__main__":
    main()
