"""Diffusion samples and inputs spread one per GPU (one process per GPU).

The structure module's sampler (upstream ``AtomDiffusion.sample``, wrapped by
the reference's ``optimized_sample``, diffusion.py:13-23) runs the 200-step
diffusion loop for ``multiplicity`` samples of one input at once.  Samples of
one input share the trunk's conditioning (s, z, the token bias) and are
otherwise independent, and so are different inputs.  This module spreads the
work units (input i, sample m) over the ranks with no collective inside the
loop:

* :func:`shard_units` gives each rank a contiguous block of units (in
  input-major order), so with one input per rank every rank runs all samples
  of its input as one batch, and with fewer inputs than ranks an input's
  samples spread over several ranks; a rank runs its units input by input,
  each input's samples as one batch (its local multiplicity);
* every sample draws all of its noise from its own generator, seeded by
  :func:`sample_seed` from (seed, input, sample), so the coordinates do not
  depend on the number of ranks or on which rank ran the sample;
* :func:`distributed_sample` gathers the coordinates of every unit onto every
  rank ([inputs, multiplicity, atoms, 3], in unit order) with one all_gather.

Upstream's sampler draws the noise of a multiplicity batch from the global
RNG; :func:`sample_upstream` keeps that API and seeds the global RNG per
(input, rank-local batch) instead, which is the one difference from an
unsharded upstream run.

:class:`EDMSampler` and :class:`TokenDiffusionModel` restate the published
sampling loop (AlphaFold 3 supplementary Algorithm 18: Karras et al. EDM noise
schedule, centre + random rotation augmentation, noise injection with gamma,
Euler step with step scale eta) and a score model built from this package's
diffusion layers (AdaLN, the bias-consuming AttentionPairBias of the token
transformer, ConditionedTransitionBlock; AF3 Algorithms 20-25 with tokens
as the atoms).  They drive the partition on hosts without upstream Boltz
(tests, ``bench.py``); with upstream installed, :func:`sample_upstream` wraps
the real sampler.
"""

import math

import torch
import torch.nn.functional as F
from torch import nn

from . import forwards, graphs, kernels, layers

__all__ = ["shard_units", "sample_seed", "distributed_sample", "sample_upstream", "EDMSampler",
           "TokenDiffusionModel", "noise_schedule", "make_denoiser"]


# ---------------------------------------------------------------------------
# Partition and gather
# ---------------------------------------------------------------------------
def unit_range(n_units, world, rank):
    """Units [begin, end) of ``rank``: contiguous blocks whose sizes differ by at most one."""
    return rank * n_units // world, (rank + 1) * n_units // world


def shard_units(n_inputs, multiplicity, world, rank):
    """The (input, sample) units of ``rank``: unit u = input * multiplicity + sample, the
    ranks owning contiguous blocks of units (:func:`unit_range`).  Returns
    {input: [samples]} in increasing order."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of world {world}")
    owned = {}
    begin, end = unit_range(n_inputs * multiplicity, world, rank)
    for unit in range(begin, end):
        owned.setdefault(unit // multiplicity, []).append(unit % multiplicity)
    return owned


def sample_seed(seed, input_index, sample_index):
    """Seed of one sample's generator (a 63-bit mix of the three integers)."""
    h = (int(seed) * 0x9E3779B97F4A7C15 + int(input_index) * 0xBF58476D1CE4E5B9
         + int(sample_index) * 0x94D049BB133111EB) & ((1 << 64) - 1)
    h ^= h >> 31
    return h & ((1 << 63) - 1)


def distributed_sample(run_samples, n_inputs, multiplicity, atoms, seed, comm, device):
    """Run this rank's units and gather every unit's coordinates onto every rank.

    ``run_samples(input_index, sample_indices, generators)`` returns the final
    coordinates [len(sample_indices), atoms, 3] (fp32) of those samples of that
    input, each sample drawing its noise from its generator.  Returns
    [n_inputs, multiplicity, atoms, 3].  The only collective is the final
    all_gather (``comm``: :class:`boltz_lumi_b200.sharded.Comm`).
    """
    world, rank = comm.world, comm.rank
    units = n_inputs * multiplicity
    per_rank = -(-units // world)  # ceil: the gather needs equal shares
    local = torch.zeros(per_rank, atoms, 3, device=device, dtype=torch.float32)
    k = 0
    for input_index, samples in shard_units(n_inputs, multiplicity, world, rank).items():
        gens = []
        for m in samples:
            g = torch.Generator(device=device)
            g.manual_seed(sample_seed(seed, input_index, m))
            gens.append(g)
        coords = run_samples(input_index, samples, gens)
        local[k:k + len(samples)] = coords
        k += len(samples)
    gathered = comm.all_gather(local)  # [world, per_rank, atoms, 3]
    out = torch.empty(units, atoms, 3, device=device, dtype=torch.float32)
    for r in range(world):
        begin, end = unit_range(units, world, r)
        out[begin:end] = gathered[r, :end - begin]
    return out.view(n_inputs, multiplicity, atoms, 3)


def sample_upstream(structure_module, inputs, multiplicity, seed, comm, **sample_kwargs):
    """Upstream ``AtomDiffusion.sample`` with the (input, sample) units spread over ranks.

    ``inputs`` is a list of keyword dicts for ``structure_module.sample`` (one per
    input: atom_mask, num_sampling_steps, network_condition_kwargs ...).  Each rank
    calls ``sample(multiplicity=<its share>)`` per input with the global RNG seeded by
    (seed, input, first local sample), and the ``sample_atom_coords`` of all units are
    gathered in unit order: [inputs, multiplicity, atoms, 3].
    """
    device = next(structure_module.parameters()).device

    def run(input_index, samples, gens):
        kwargs = dict(inputs[input_index])
        kwargs.update(sample_kwargs)
        torch.manual_seed(sample_seed(seed, input_index, samples[0]))
        out = structure_module.sample(multiplicity=len(samples), **kwargs)
        return out["sample_atom_coords"].float().reshape(len(samples), -1, 3)

    atoms = int(inputs[0]["atom_mask"].shape[-1])
    return distributed_sample(run, len(inputs), multiplicity, atoms, seed, comm, device)


# ---------------------------------------------------------------------------
# A sampler and score model on this package's diffusion layers
# ---------------------------------------------------------------------------
def noise_schedule(steps, sigma_data=16.0, s_max=160.0, s_min=4e-4, rho=7.0, device=None):
    """The EDM noise levels c_0 > ... > c_steps = 0 used by AF3 Algorithm 18."""
    t = torch.arange(steps + 1, dtype=torch.float64, device=device) / steps
    levels = sigma_data * (s_max ** (1 / rho) + t * (s_min ** (1 / rho) - s_max ** (1 / rho))) ** rho
    levels[-1] = 0.0
    return levels.float()


def _random_rotations(generators, device):
    """Uniform random rotations [S, 3, 3], one per generator, from normalised Gaussian
    quaternions (device-side, no host synchronisation; the matrix algebra is batched)."""
    q = torch.stack([torch.randn(4, generator=g, device=device) for g in generators])
    w, x, y, z = (q / q.norm(dim=1, keepdim=True)).unbind(1)
    return torch.stack([1 - 2 * (y * y + z * z), 2 * (x * y - z * w), 2 * (x * z + y * w),
                        2 * (x * y + z * w), 1 - 2 * (x * x + z * z), 2 * (y * z - x * w),
                        2 * (x * z - y * w), 2 * (y * z + x * w), 1 - 2 * (x * x + y * y)], 1).view(-1, 3, 3)


class EDMSampler:
    """AF3 supplementary Algorithm 18 (SampleDiffusion) for a batch of samples of one input.

    Every random draw of sample m comes from ``generators[m]``.
    """

    def __init__(self, steps=200, sigma_data=16.0, gamma_0=0.8, gamma_min=1.0, noise_scale=1.003,
                 step_scale=1.5, s_trans=1.0):
        self.steps, self.sigma_data = steps, sigma_data
        self.gamma_0, self.gamma_min, self.noise_scale = gamma_0, gamma_min, noise_scale
        self.step_scale, self.s_trans = step_scale, s_trans

    def _noise(self, generators, shape, device):
        return torch.stack([torch.randn(shape, generator=g, device=device) for g in generators])

    def _augment(self, x, generators):
        x = x - x.mean(dim=1, keepdim=True)
        rots = _random_rotations(generators, x.device)
        trans = self._noise(generators, (1, 3), x.device) * self.s_trans
        return torch.einsum("sij,snj->sni", rots, x) + trans

    def sample(self, denoise, atoms, generators, device):
        """``denoise(x_noisy [S, atoms, 3], sigma [S])`` -> denoised coordinates."""
        levels = noise_schedule(self.steps, self.sigma_data, device=device).tolist()
        x = levels[0] * self._noise(generators, (atoms, 3), device)
        for c_prev, c in zip(levels[:-1], levels[1:]):
            x = self._augment(x, generators)
            gamma = self.gamma_0 if c > self.gamma_min else 0.0
            t_hat = c_prev * (gamma + 1)
            eps = self.noise_scale * math.sqrt(max(t_hat ** 2 - c_prev ** 2, 0.0)) * \
                self._noise(generators, (atoms, 3), device)
            x_noisy = x + eps
            sigma = torch.full((len(generators),), t_hat, device=device)
            x_denoised = denoise(x_noisy, sigma)
            delta = (x_noisy - x_denoised) / t_hat
            x = x_noisy + self.step_scale * (c - t_hat) * delta
        return x


class TokenDiffusionModel(nn.Module):
    """Score model: EDM preconditioning around a token transformer of this package's layers.

    Per layer (AF3 Algorithms 23-25 with tokens as atoms): a += sigmoid(W_g s) *
    AttentionPairBias(AdaLN(a, s), bias_l); a += ConditionedTransitionBlock(a, s).  The
    attention takes the layer's slice of the prepared token bias [1, N, N, L*H] and the
    samples of the batch share it (multiplicity without a copy).  s = W_s s_trunk + W_t
    Fourier(sigma); a = W_r (c_in x) + s.  Output: x_denoised = c_skip x + c_out W_o LN(a).
    """

    def __init__(self, depth=24, c_token=768, c_s=384, heads=16, sigma_data=16.0, fourier=256):
        super().__init__()
        self.depth, self.c_token, self.heads, self.sigma_data = depth, c_token, heads, sigma_data
        self.s_in = nn.Linear(c_s, c_token, bias=False)
        self.t_in = nn.Linear(fourier, c_token, bias=False)
        self.r_in = nn.Linear(3, c_token, bias=False)
        self.register_buffer("fourier_w", torch.randn(fourier, generator=torch.Generator().manual_seed(7)))
        self.register_buffer("fourier_b", torch.rand(fourier, generator=torch.Generator().manual_seed(8)))
        self.adaln = nn.ModuleList([layers.AdaLN(c_token, c_token) for _ in range(depth)])
        self.attention = nn.ModuleList([layers.AttentionPairBias(c_token, num_heads=heads, inf=1e6,
                                                                 compute_pair_bias=False) for _ in range(depth)])
        self.gate = nn.ModuleList([nn.Linear(c_token, c_token) for _ in range(depth)])
        self.transition = nn.ModuleList([layers.ConditionedTransitionBlock(c_token, c_token) for _ in range(depth)])
        self.out_norm = nn.LayerNorm(c_token)
        self.r_out = nn.Linear(c_token, 3, bias=False)

    def conditioning(self, s_trunk):
        """The sigma-independent part of s (computed once per input)."""
        return forwards._linear32(self, "_bl_w3_s_in", s_trunk, [self.s_in.weight])

    def forward(self, x_noisy, sigma, s_base, bias, mask):
        """x_noisy [S, N, 3], sigma [S], s_base [1, N, c], bias [1, N, N, L*H], mask [1, N] -> [S, N, 3]."""
        samples, n = x_noisy.shape[0], x_noisy.shape[1]
        sd = self.sigma_data
        var = sigma * sigma + sd * sd
        c_in, c_skip, c_out = var.rsqrt(), sd * sd / var, sigma * sd * var.rsqrt()
        c_noise = torch.log(sigma / sd) * 0.25
        fourier = torch.cos(2 * math.pi * (c_noise[:, None] * self.fourier_w + self.fourier_b))
        t_emb = forwards._linear32(self, "_bl_w3_t_in", fourier, [self.t_in.weight])  # [S, c]
        s = (s_base + t_emb[:, None, :]).contiguous()  # [S, N, c]
        a = (F.linear(x_noisy * c_in[:, None, None], self.r_in.weight) + s).contiguous()
        mask_s = mask.expand(samples, n).contiguous()
        h = self.heads
        for layer in range(self.depth):
            b = self.adaln[layer](a, s)
            att = self.attention[layer]
            bias_l = bias[..., layer * h:(layer + 1) * h]
            o = forwards.token_attention_forward(att, b, bias_l, mask_s, b, multiplicity=samples)
            g = forwards._linear32(self, f"_bl_w3_gate{layer}", s, [self.gate[layer].weight], [self.gate[layer].bias])
            a = a + kernels.epilogue(g.contiguous(), o.contiguous(), None, kernels.GATE)
            a = a + self.transition[layer](a, s)
        an = kernels.layer_norm(a, self.out_norm.weight, self.out_norm.bias, self.out_norm.eps,
                                out_dtype=torch.float32)
        r = F.linear(an, self.r_out.weight)
        return c_skip[:, None, None] * x_noisy + c_out[:, None, None] * r


def make_denoiser(model, s_trunk, bias, mask, cuda_graphs=True):
    """``denoise(x, sigma)`` of one input for :class:`EDMSampler`.  The sigma-independent
    conditioning is computed once; with ``cuda_graphs`` the score model replays from a CUDA
    graph from its third call on (:class:`boltz_lumi_b200.graphs.GraphedStep`: x and sigma are
    copied into the graph's buffers, the conditioning is read in place), which removes the
    host launch overhead of the ~500 kernels of a 24-layer step."""
    s_base = model.conditioning(s_trunk)
    fn = graphs.GraphedStep(model.forward) if cuda_graphs else model.forward
    return lambda x, sigma: fn(x, sigma, s_base, bias, mask)


def synthetic_conditioning(n_tokens, depth, heads, c_s=384, seed=0, device="cuda"):
    """Seeded stand-ins for the trunk outputs one input conditions the sampler on:
    s_trunk [1, N, c_s] ~ N(0, 1), the prepared token bias [1, N, N, L*H] ~ N(0, 1)
    (head-major storage, as the reference's prepare_token_bias packs it), mask ones."""
    g = torch.Generator().manual_seed(seed)
    s_trunk = torch.randn(1, n_tokens, c_s, generator=g).to(device)
    bias = torch.randn(1, depth * heads, n_tokens, n_tokens, generator=g).to(device).permute(0, 2, 3, 1)
    mask = torch.ones(1, n_tokens, device=device)
    return s_trunk, bias, mask


def seeded_model(depth=24, c_token=768, heads=16, c_s=384, seed=0, device="cuda"):
    """A TokenDiffusionModel with seeded N(0, 1/fan_in) weights (unit-mean norm weights)."""
    model = TokenDiffusionModel(depth=depth, c_token=c_token, c_s=c_s, heads=heads)
    g = torch.Generator().manual_seed(seed)
    with torch.no_grad():
        for name, p in model.named_parameters():
            if p.dim() == 2:
                p.copy_(torch.randn(p.shape, generator=g) * p.shape[1] ** -0.5)
            elif "norm" in name and name.endswith("weight"):
                p.fill_(1.0)
            else:
                p.zero_()
    return model.to(device).eval()
