"""Run the Boltz CLI with the B200 pair-path kernels:

    python -m boltz_lumi_b200 predict input.yaml [boltz predict options]

Mirrors the reference's wrapper (__main__.py:33-52): check the supported Boltz
version, then run ``boltz.main.cli`` with ``Trainer.predict`` patched so that
an inference callback installs the kernels on the model before prediction
and rejects failed or non-finite predictions afterwards.  Upstream Boltz,
PyTorch Lightning and their dependencies must be installed; this package does
not vendor them.
"""

import sys
from importlib.metadata import PackageNotFoundError, version
from unittest.mock import patch

import torch

from . import SUPPORTED_BOLTZ_VERSION
from .adapters import install

_CHECKED_OUTPUTS = ("coords", "confidence_score", "affinity_pred_value", "affinity_probability_binary")


def _callback_class():
    from pytorch_lightning import Callback

    class InferenceAdapter(Callback):
        """Installs the kernels at predict start; checks each batch's outputs."""

        def __init__(self, optimize=True):
            self.optimize = optimize

        def on_predict_start(self, trainer, model):
            if self.optimize and model.device.type == "cuda":
                install(model)

        def on_predict_batch_end(self, trainer, model, outputs, batch, batch_idx, dataloader_idx=0):
            if outputs.get("exception"):
                raise RuntimeError("Boltz prediction failed; see the preceding log")
            for key in _CHECKED_OUTPUTS:
                if key in outputs and not torch.isfinite(outputs[key]).all():
                    raise RuntimeError(f"non-finite prediction output: {key}")

    return InferenceAdapter


def run(arguments=None, optimize=True):
    try:
        installed = version("boltz")
    except PackageNotFoundError as err:
        raise RuntimeError(f"boltz=={SUPPORTED_BOLTZ_VERSION} is required for `predict`") from err
    if installed != SUPPORTED_BOLTZ_VERSION:
        raise RuntimeError(f"this adapter supports Boltz {SUPPORTED_BOLTZ_VERSION}, found {installed}")
    from boltz.main import cli
    from pytorch_lightning import Trainer

    arguments = list(sys.argv[1:] if arguments is None else arguments)
    adapter_cls = _callback_class()
    original_predict = Trainer.predict

    def predict(trainer, model, *args, **kwargs):
        adapter = adapter_cls(optimize)
        trainer.callbacks.append(adapter)
        try:
            return original_predict(trainer, model, *args, **kwargs)
        finally:
            trainer.callbacks.remove(adapter)

    with patch.object(Trainer, "predict", predict):
        return cli(arguments, standalone_mode=False)


if __name__ == "__main__":
    run()
