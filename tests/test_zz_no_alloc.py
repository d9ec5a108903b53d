"""The allocation-free pair transition (bl_pair_transition_static).

Some hosts may not allocate device memory while they run inference (they keep
all of HBM in their own pool, or their plugin interface passes a kernel only
its inputs and outputs).  bl_pair_transition_static serves them: it keeps its
intermediates in a fixed array inside the library.  This test calls it through
the C ABI on two calls in a row (the second call reuses the array the first one
left behind) and checks each result against the CPU oracle's bf16-autocast
Transition and against the library's allocating pair-transition entry point.

The file name sorts last so that a run stopping at the first failure has
already run every other test.
"""

import ctypes

import pytest
import torch

from conftest import assert_close

pytestmark = pytest.mark.gpu

MAX_ROWS = 1024


def _transition(seed):
    from boltz_lumi_b200 import layers

    g = torch.Generator().manual_seed(seed)
    module = layers.Transition(128, 512)
    with torch.no_grad():
        for name, p in module.named_parameters():
            mean = 1.0 if name.endswith("norm.weight") else 0.0
            p.copy_(torch.randn(p.shape, generator=g) * 0.05 + mean)
    return module.cuda().eval()


def _static_call(module, x):
    from boltz_lumi_b200 import _lib

    w12 = torch.cat([module.fc1.weight, module.fc2.weight], 0).bfloat16().contiguous()
    w3 = module.fc3.weight.bfloat16().contiguous()
    out = torch.empty(x.shape[0], 128, device=x.device, dtype=torch.bfloat16)
    lib = _lib.load()
    status = lib.bl_pair_transition_static(
        x.data_ptr(), x.shape[0], module.norm.weight.data_ptr(), module.norm.bias.data_ptr(),
        ctypes.c_float(module.norm.eps), w12.data_ptr(), w3.data_ptr(), out.data_ptr(),
        torch.cuda.current_stream().cuda_stream)
    assert status == 0, lib.bl_last_error().decode()
    return out


def test_static_transition_matches_allocating_path_twice():
    import oracle
    from boltz_lumi_b200 import forwards

    module = _transition(seed=5)
    ref = oracle.Transition(128, 512)
    ref.load_state_dict({k: v.cpu() for k, v in module.state_dict().items()})
    with torch.inference_mode():
        for call, rows in enumerate((MAX_ROWS, 300)):
            g = torch.Generator().manual_seed(100 + call)
            x = torch.randn(rows, 128, generator=g)
            xc = x.cuda()
            # forwards.transition_forward runs the fused single-kernel transition
            # (bl_pair_transition) at 128 -> 512 -> 128.  It keeps the same bf16
            # rounding points (LN, fc1|fc2, SiLU product) as the static path's
            # four kernels and differs only in fp32 accumulation order, so the
            # two agree to one bf16 ulp.
            expected = forwards.transition_forward(module, xc)
            actual = _static_call(module, xc)
            torch.cuda.synchronize()
            assert_close(actual.float(), expected.float(), atol=1e-6, rtol=2.0 ** -7)
            # Independent check: the oracle's bf16-autocast restatement, per-op bound 2e-2.
            assert_close(actual.float(), ref(x), atol=2e-2)


def test_static_transition_rejects_too_many_rows():
    from boltz_lumi_b200 import _lib

    lib = _lib.load()
    status = lib.bl_pair_transition_static(None, MAX_ROWS + 1, None, None, ctypes.c_float(1e-5), None, None, None,
                                           None)
    assert status == 1
    assert b"scratch limit" in lib.bl_last_error()
