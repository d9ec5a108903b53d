"""Install the B200 pair-path forwards on a Boltz-2 model (the drop-in boundary).

Mirrors the reference's ``install(model)`` (adapters.py:7-47): walk
``model.named_modules()`` and rebind ``forward`` methods by class name and
module path with ``types.MethodType``.  The rebound forwards fall back to the
module's original class forward (upstream's eager code) only where upstream
itself needs it -- autograd / training mode, or shapes the kernels do not
cover (for example the template module's narrower pair width) -- exactly as
the reference does; they never fall back to a CPU path.
"""

import contextlib
from types import MethodType

import torch

from . import atom_conditioning, forwards, graphs

_TRIANGLE_ATTENTION = {"TriangleAttention", "TriangleAttentionEndingNode"}
_TRIANGLE_MULTIPLICATION = {"TriangleMultiplicationIncoming", "TriangleMultiplicationOutgoing"}
_DIFFUSION = {"AdaLN", "ConditionedTransitionBlock"}


def device_supported(device=None):
    """The kernels are built for sm_100a (B200)."""
    if not torch.cuda.is_available():
        return False
    major, minor = torch.cuda.get_device_capability(device)
    return (major, minor) == (10, 0)


def _inference(module, *tensors):
    return (not module.training and not torch.is_grad_enabled()
            and all(t is None or t.is_cuda for t in tensors))


def _bf16_autocast():
    """The trunk kernels implement upstream's bf16-autocast contract (as the
    reference requires, multiplication.py:61-62, triangle.py:156-159)."""
    return torch.is_autocast_enabled("cuda") and torch.get_autocast_dtype("cuda") == torch.bfloat16


def _fp32_mode(x):
    """Autocast off and fp32 input: upstream computes the whole op in fp32 (the
    reference's fast path takes this case too, triangle.py:47-51)."""
    return not torch.is_autocast_enabled("cuda") and x.dtype == torch.float32


def _triangle_attention(self, x, mask=None, chunk_size=None, use_kernels=False):
    cls = type(self)
    fp32 = _fp32_mode(x)
    if (use_kernels or not _inference(self, x, mask) or not (_bf16_autocast() or fp32) or x.dim() != 4
            or x.shape[-1] != 128 or not forwards._attention_supported(self) or x.shape[1] > 4096):
        return cls.forward(self, x, mask=mask, chunk_size=chunk_size, use_kernels=use_kernels)
    starting = getattr(self, "starting", cls.__name__ != "TriangleAttentionEndingNode")
    self.starting = starting
    if fp32:
        return forwards.triangle_attention_forward_fp32(self, x, mask, chunk_size)
    return forwards.triangle_attention_forward(self, x.float(), mask, chunk_size)


def _triangle_multiplication(self, x, mask, use_kernels=False):
    cls = type(self)
    if (use_kernels or not _inference(self, x, mask) or not _bf16_autocast() or x.dim() != 4
            or x.shape[-1] != 128 or self.p_in.weight.shape != (256, 128) or self.p_in.bias is not None):
        return cls.forward(self, x, mask, use_kernels=use_kernels)
    self.outgoing = cls.__name__ == "TriangleMultiplicationOutgoing"
    return forwards.triangle_multiplication_forward(self, x.float(), mask)


def _pair_transition(self, x, chunk_size=None):
    cls = type(self)
    if (chunk_size is not None or not _inference(self, x) or not _bf16_autocast() or x.shape[-1] % 8
            or self.fc1.weight.shape[0] % 64 or any(f.bias is not None for f in (self.fc1, self.fc2, self.fc3))):
        return cls.forward(self, x, chunk_size=chunk_size)
    return forwards.transition_forward(self, x.float())


def _adaln(self, a, s):
    if (not _inference(self, a, s) or torch.is_autocast_enabled("cuda") or a.dtype != torch.float32
            or s.dtype != torch.float32 or a.shape[-1] % 4 or a.shape[-1] > 2048):
        return type(self).forward(self, a, s)
    return forwards.adaln_forward(self, a.contiguous(), s.contiguous())


def _conditioned_transition(self, a, s):
    if (not _inference(self, a, s) or torch.is_autocast_enabled("cuda") or a.dtype != torch.float32
            or s.dtype != torch.float32 or a.shape[-1] % 4 or a.shape[-1] > 2048):
        return type(self).forward(self, a, s)
    return forwards.conditioned_transition_forward(self, a.contiguous(), s.contiguous())


def _token_attention(self, s, z, mask, k_in, multiplicity=1):
    cls = type(self)
    if (not _inference(self, s, z, mask, k_in) or self.compute_pair_bias or torch.is_autocast_enabled("cuda")):
        return cls.forward(self, s, z, mask, k_in, multiplicity)
    bias = self.proj_z(z)
    if (not forwards.token_attention_supported(self, s, k_in, bias, mask)
            or bias.shape[0] * multiplicity not in (s.shape[0], 1)):
        return cls.forward(self, s, z, mask, k_in, multiplicity)
    return forwards.attend_with_bias(self, s, bias, mask, k_in)


def _sample(self, *args, **kwargs):
    """``AtomDiffusion.sample`` with the token-transformer bias packed dense
    once per prediction and, for one input and one sample, the atom
    conditioning projections computed once for all steps (the reference's
    optimized_sample, diffusion.py:13-23)."""
    sample = type(self).sample
    conditioning = kwargs.get("diffusion_conditioning")
    if torch.is_grad_enabled() or self.training or not conditioning or "token_trans_bias" not in conditioning:
        return sample(self, *args, **kwargs)
    conditioning = dict(conditioning)
    conditioning["token_trans_bias"] = forwards.prepare_token_bias(conditioning["token_trans_bias"])
    kwargs["diffusion_conditioning"] = conditioning
    context = contextlib.nullcontext()
    single = "c" in conditioning and conditioning["c"].shape[0] == 1
    if kwargs.get("multiplicity", 1) == 1 and single and hasattr(getattr(self, "score_model", None),
                                                                   "atom_attention_encoder"):
        context = atom_conditioning.atom_conditioning_cache(self.score_model)
    with context, _graphed_score_model(self):
        return sample(self, *args, **kwargs)


@contextlib.contextmanager
def _graphed_score_model(structure):
    """With ``install(model, cuda_graphs=True)``: the score model's forward
    replays a CUDA graph from the third diffusion step on, for this sampling
    call only (features and conditioning change between predictions)."""
    score_model = getattr(structure, "score_model", None)
    if not getattr(structure, "_b200_cuda_graphs", False) or score_model is None or "forward" in score_model.__dict__:
        yield
        return
    step = graphs.GraphedStep(score_model.forward)
    score_model.forward = step
    try:
        yield
    finally:
        del score_model.forward
        step.reset()


def install(model, require_device=True, cuda_graphs=False):
    """Rebind the hot-path forwards of ``model`` in place; idempotent.

    Returns the number of modules rebound.  Like the reference, modules are
    matched by class name: every TriangleAttention / TriangleAttentionEndingNode
    and TriangleMultiplication{Incoming,Outgoing}, every ``*.transition_z``
    Transition, the AdaLN / ConditionedTransitionBlock modules under
    ``structure_module.score_model`` and the AttentionPairBias modules under
    ``structure_module.score_model.token_transformer``; and, like the
    reference (adapters.py:46), wraps ``structure_module.sample`` so the token
    bias is packed once per prediction.  ``cuda_graphs=True`` additionally
    replays the score model of each sampling call from a CUDA graph
    (:mod:`boltz_lumi_b200.graphs`); it needs a capture-safe score model and is
    off by default.
    """
    if getattr(model, "_b200_optimized", False):
        return 0
    if require_device and not device_supported():
        return 0
    count = 0
    for name, module in model.named_modules():
        cls = type(module).__name__
        if cls in _TRIANGLE_ATTENTION:
            module.forward = MethodType(_triangle_attention, module)
            count += 1
        elif cls in _TRIANGLE_MULTIPLICATION:
            module.forward = MethodType(_triangle_multiplication, module)
            count += 1
        elif cls == "Transition" and name.endswith("transition_z"):
            module.forward = MethodType(_pair_transition, module)
            count += 1
        elif cls in _DIFFUSION and name.startswith("structure_module.score_model."):
            module.forward = MethodType(_adaln if cls == "AdaLN" else _conditioned_transition, module)
            count += 1
        elif cls == "AttentionPairBias" and name.startswith("structure_module.score_model.token_transformer."):
            module.forward = MethodType(_token_attention, module)
            count += 1
    structure = getattr(model, "structure_module", None)
    if structure is not None and callable(getattr(type(structure), "sample", None)):
        structure.sample = MethodType(_sample, structure)
        structure._b200_cuda_graphs = bool(cuda_graphs)
    model._b200_optimized = True
    return count


def uninstall(model):
    """Restore the class forwards rebound by :func:`install`."""
    for _, module in model.named_modules():
        if "forward" in module.__dict__ and getattr(module.forward, "__func__", None) in (
                _triangle_attention, _triangle_multiplication, _pair_transition, _adaln, _conditioned_transition,
                _token_attention):
            del module.forward
    structure = getattr(model, "structure_module", None)
    if structure is not None and getattr(structure.__dict__.get("sample"), "__func__", None) is _sample:
        del structure.sample
        structure.__dict__.pop("_b200_cuda_graphs", None)
    model._b200_optimized = False
