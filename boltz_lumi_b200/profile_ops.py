"""Run one pair-path op (or a whole Pairformer block) a few times, for profilers.

    python -m boltz_lumi_b200.profile_ops --op att_start --n 512 --iters 3

Ops: tri_mul_out, tri_mul_in, att_start, att_end, transition, block, c2
(att_start + att_end), c3 (tri_mul_out + tri_mul_in + transition), and the
diffusion token transformer's attention: token_attention (the whole
AttentionPairBias forward, c_s 768, 16 heads, a layer of a prepared 24-layer
token bias, --mult samples) and token_core (bl_token_attention alone); and
linear (the fp32 tensor-core linear bl_linear_split3 at --m x --n x --k).  Inputs
and weights are the benchmark's synthetic ones (seeded); z is updated in
place like in the Pairformer block.  Prints the mean device time per call.
"""

import argparse

import torch

from . import forwards, kernels, layers


def seeded_block(seed=1234):
    module = layers.PairformerLayer()
    g = torch.Generator().manual_seed(seed)
    with torch.no_grad():
        for name, p in module.named_parameters():
            mean = 1.0 if "norm" in name and name.endswith("weight") else 0.0
            p.copy_(torch.randn(p.shape, generator=g) * (1.0 / 128) ** 0.5 + mean)
    return module.eval()


def _token_ops(n, mult, layers_=24, heads=16, c_s=768):
    torch.manual_seed(3)
    module = layers.AttentionPairBias(c_s, num_heads=heads, compute_pair_bias=False).cuda().eval()
    g = torch.Generator().manual_seed(9)
    s = torch.randn(mult, n, c_s, generator=g).cuda()
    raw = torch.randn(1, n, n, layers_ * heads, generator=g).cuda()
    bias = forwards.prepare_token_bias(raw).view(1, n, n, layers_, heads)[:, :, :, 0]
    del raw
    mask = torch.ones(mult, n, device="cuda")
    d = c_s // heads
    q, k, v, gate = (torch.randn(mult, n, heads, d, generator=g).cuda() for _ in range(4))
    return {
        "token_attention": lambda: module(s, bias, mask, s, multiplicity=mult),
        "token_core": lambda: kernels.token_attention(q, k, v, bias.permute(0, 3, 1, 2), mask, 1e6, gate=gate),
    }


def main():
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("--op", default="block",
                        choices=["tri_mul_out", "tri_mul_in", "att_start", "att_end", "transition", "block",
                                 "token_attention", "token_core", "linear", "c2", "c3"])
    parser.add_argument("--n", type=int, default=512)
    parser.add_argument("--iters", type=int, default=3)
    parser.add_argument("--mult", type=int, default=1, help="diffusion samples (token ops)")
    parser.add_argument("--masked-tail", type=float, default=0.0,
                        help="fraction of tokens masked at the end (rows and columns of the pair mask)")
    parser.add_argument("--m", type=int, default=117, help="rows (linear)")
    parser.add_argument("--k", type=int, default=768, help="input features (linear)")
    parser.add_argument("--n-out", type=int, default=768, help="output features (linear)")
    args = parser.parse_args()
    block = seeded_block().cuda()
    g = torch.Generator().manual_seed(7)
    n = args.n
    z = torch.randn(1, n, n, 128, generator=g).cuda()
    s = torch.randn(1, n, 384, generator=g).cuda()
    mask = torch.ones(1, n, device="cuda")
    pmask = torch.ones(1, n, n, device="cuda")
    tail = int(round(args.masked_tail * n))
    if tail:
        mask[:, n - tail:] = 0
        pmask[:, n - tail:, :] = 0
        pmask[:, :, n - tail:] = 0
    ops = {
        "tri_mul_out": lambda: forwards.triangle_multiplication_forward(block.tri_mul_out, z, pmask, residual=z),
        "tri_mul_in": lambda: forwards.triangle_multiplication_forward(block.tri_mul_in, z, pmask, residual=z),
        "att_start": lambda: forwards.triangle_attention_forward(block.tri_att_start, z, pmask, residual=z),
        "att_end": lambda: forwards.triangle_attention_forward(block.tri_att_end, z, pmask, residual=z),
        "transition": lambda: forwards.transition_forward(block.transition_z, z, residual=z),
        "block": lambda: block(s, z, mask, pmask),
    }
    # Composite measurement configs: c2 = both triangle attentions, c3 = both
    # triangle multiplications and the pair transition.
    ops["c2"] = lambda: (ops["att_start"](), ops["att_end"]())
    ops["c3"] = lambda: (ops["tri_mul_out"](), ops["tri_mul_in"](), ops["transition"]())
    if args.op.startswith("token"):
        ops.update(_token_ops(n, args.mult))
    if args.op == "linear":
        x = torch.randn(args.m, args.k, generator=g).cuda()
        w3 = kernels.split3((torch.randn(args.n_out, args.k, generator=g) * args.k ** -0.5).cuda())
        x3 = kernels.split3(x)
        ops["linear"] = lambda: kernels.linear_f32(x, w3, x3=x3)
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
    shape = f"m={args.m} n={args.n_out} k={args.k}" if args.op == "linear" else f"n={n}"
    print(f"{args.op} {shape}: {start.elapsed_time(end) / args.iters:.4f} ms per call")


if __name__ == "__main__":
    main()
