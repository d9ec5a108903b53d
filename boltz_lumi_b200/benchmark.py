"""Upstream-versus-optimized benchmark of a Boltz-2 model, with stage timings.

    python -m boltz_lumi_b200.benchmark predict input.yaml [boltz predict options] [--repeats 3]

Follows the reference's harness (benchmark.py:20-240):

- The same preprocessed inputs are predicted first with upstream's eager modules, then after
  :func:`boltz_lumi_b200.adapters.install`, each for ``repeats + 1`` rounds with the same seed.
- Round 0 of each recipe is the cold one.
- Each model call records its wall time (device-synchronised), peak memory and the device
  time of the model's stages (CUDA events around ``input_embedder``, ``template_module``,
  ``msa_module``, ``pairformer_module``, ``diffusion_conditioning``, ``confidence_module``
  and ``structure_module.sample``).
- Every optimized output field is compared with the upstream output of the same input.
- ``timings.json`` holds the settings, every call and round, the per-field errors, the warm
  means of both recipes and the time saved.

This build is not bitwise identical to upstream: it matches it within the end-to-end
tolerances this package targets. So the comparison reports errors per field and judges them against
:data:`TOLERANCES`, where the reference asks for atol = rtol = 0:

- coordinate RMSD <= 0.1 Angstrom;
- pLDDT within 0.01.

The other fields are recorded without a bound.

:func:`compare` is the harness itself and works on any model with those module names.
:func:`main` drives it through the upstream ``boltz predict`` CLI, which needs upstream Boltz
and PyTorch Lightning installed.
"""

import argparse
import json
import statistics
import sys
import time
from contextlib import contextmanager
from pathlib import Path

import torch

from . import adapters

STAGES = ("input_embedder", "template_module", "msa_module", "pairformer_module", "diffusion_conditioning",
          "confidence_module")
OUTPUT_FIELDS = ("coords", "plddt", "confidence_score", "ptm", "iptm", "complex_plddt", "ligand_iptm",
                 "protein_iptm", "affinity_pred_value", "affinity_probability_binary")
# field -> (metric, bound): the end-to-end tolerances of the pair-path build.
TOLERANCES = {"coords": ("rmsd", 0.1), "plddt": ("max_abs", 0.01)}


@contextmanager
def stage_timers(model, events):
    """Append (stage, start, end) CUDA events for every call of a stage module
    (matched by name) and of ``structure_module.sample`` while open."""
    saved = []

    def wrap(owner, attribute, name):
        original = getattr(owner, attribute)
        saved.append((owner, attribute, attribute in owner.__dict__, original))

        def timed(*args, **kwargs):
            start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            start.record()
            try:
                with torch.profiler.record_function(name):
                    return original(*args, **kwargs)
            finally:
                end.record()
                events.append((name, start, end))

        setattr(owner, attribute, timed)

    try:
        for name, module in model.named_modules():
            if name in STAGES:
                wrap(module, "forward", name)
        sampler = getattr(model, "structure_module", None)
        if sampler is not None and callable(getattr(sampler, "sample", None)):
            wrap(sampler, "sample", "diffusion_sample")
        yield
    finally:
        for owner, attribute, had, original in reversed(saved):
            if had:
                setattr(owner, attribute, original)
            else:
                delattr(owner, attribute)


def field_error(field, value, expected):
    """Error record of one output field against the upstream value."""
    value, expected = value.double(), expected.double()
    delta = value - expected
    norm = expected.norm().item()
    record = dict(field=field, max_absolute_error=delta.abs().max().item() if delta.numel() else 0.0,
                  relative_l2_error=delta.norm().item() / norm if norm else None,
                  differing_values=int((value != expected).sum()))
    if field == "coords" and value.shape[-1] == 3 and value.numel():
        record["rmsd"] = delta.pow(2).sum(-1).mean().sqrt().item()
    metric, bound = TOLERANCES.get(field, (None, None))
    if metric is not None:
        measured = record.get(metric, record["max_absolute_error"] if metric == "max_abs" else None)
        record.update(metric=metric, bound=bound, within_bound=measured is not None and measured <= bound)
    return record


def _outputs(output):
    return {k: output[k].detach().cpu() for k in OUTPUT_FIELDS if isinstance(output.get(k), torch.Tensor)}


def compare(model, predict_once, inputs, repeats=3, seed=42, output=None, settings=None,
            install=adapters.install, uninstall=adapters.uninstall):
    """Run ``predict_once(model, item)`` for every input: upstream first, then
    with the kernels installed; ``repeats + 1`` rounds each, same seed per call.

    ``inputs`` is a list of (candidate_id, item).  Returns the report (also
    written to ``output / "timings.json"`` when ``output`` is given).  The
    model is left as it was found (``uninstall`` after the optimized rounds).
    """
    if repeats < 1:
        raise ValueError("use at least one warm repeat")
    report = dict(settings or {}, torch=torch.__version__, cuda=torch.version.cuda,
                  gpu=torch.cuda.get_device_name(0), repeats=repeats, seed=seed, tolerances=TOLERANCES,
                  model_calls=[], rounds=[], errors=[], status="running")
    references = {}
    events = []

    def save():
        if output is not None:
            Path(output).mkdir(parents=True, exist_ok=True)
            (Path(output) / "timings.json").write_text(json.dumps(report, indent=2) + "\n")

    def call(recipe, iteration, candidate, item):
        torch.manual_seed(seed)
        events.clear()
        torch.cuda.synchronize()
        torch.cuda.reset_peak_memory_stats()
        begin = time.perf_counter()
        result = predict_once(model, item)
        torch.cuda.synchronize()
        elapsed = time.perf_counter() - begin
        stages = {}
        for name, start, end in events:
            stages[name] = stages.get(name, 0.0) + start.elapsed_time(end) / 1000
        current = dict(recipe=recipe, iteration=iteration, first=iteration == 0, candidate=candidate)
        report["model_calls"].append(dict(current, model_s=elapsed,
                                          peak_allocated_bytes=torch.cuda.max_memory_allocated(),
                                          stages_s=stages))
        values = _outputs(result)
        if any(not torch.isfinite(v).all() for v in values.values()):
            raise RuntimeError(f"non-finite prediction for {candidate} ({recipe})")
        expected = references.setdefault(candidate, values)
        for field, value in values.items():
            report["errors"].append(dict(current, **field_error(field, value, expected[field])))

    try:
        for recipe in ("upstream", "optimized"):
            if recipe == "optimized":
                install(model)
            try:
                with stage_timers(model, events):
                    for iteration in range(repeats + 1):
                        begin = time.perf_counter()
                        for candidate, item in inputs:
                            call(recipe, iteration, candidate, item)
                        report["rounds"].append(dict(recipe=recipe, iteration=iteration,
                                                     candidates=[c for c, _ in inputs],
                                                     round_s=time.perf_counter() - begin))
                        save()
            finally:
                if recipe == "optimized":
                    uninstall(model)
        summarize(report)
    except BaseException as error:
        report.update(status="failed", error=str(error))
        raise
    finally:
        save()
    return report


def summarize(report):
    """Warm means per recipe, time saved, stage means and the status."""
    for recipe in ("upstream", "optimized"):
        warm = [c for c in report["model_calls"] if c["recipe"] == recipe and not c["first"]]
        if warm:
            report[recipe + "_warm_mean_s"] = statistics.mean(c["model_s"] for c in warm)
            names = sorted({n for c in warm for n in c["stages_s"]})
            report[recipe + "_warm_stages_s"] = {
                n: statistics.mean(c["stages_s"].get(n, 0.0) for c in warm) for n in names}
    if "upstream_warm_mean_s" in report and "optimized_warm_mean_s" in report:
        upstream = report["upstream_warm_mean_s"]
        saved = upstream - report["optimized_warm_mean_s"]
        report.update(saved_s=saved, saved_percent=100 * saved / upstream if upstream else None,
                      speedup=upstream / report["optimized_warm_mean_s"] if report["optimized_warm_mean_s"] else None)
    failed = [e for e in report["errors"] if e.get("within_bound") is False]
    report["status"] = "outside_tolerance" if failed else "complete"
    return report


def main(argv=None):
    """``boltz predict`` twice (upstream, then optimized) on the same inputs."""
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter,
                                     allow_abbrev=False)
    parser.add_argument("--repeats", type=int, default=3)
    parser.add_argument("--output", type=Path, default=None, help="report folder (default: <out_dir>/benchmark)")
    args, arguments = parser.parse_known_args(sys.argv[1:] if argv is None else argv)
    try:
        from boltz.main import cli
        from pytorch_lightning import Trainer
    except ImportError as err:
        raise SystemExit(f"the benchmark drives upstream `boltz predict`: install boltz and pytorch_lightning ({err})")
    if torch.cuda.device_count() != 1:
        raise SystemExit("run the comparison with one visible GPU")
    if arguments[:1] == ["predict"]:
        arguments.pop(0)
    original_predict = Trainer.predict

    def predict(trainer, model, *positional, **keywords):
        datamodule = keywords.get("datamodule")
        batches = list(datamodule.predict_dataloader())
        inputs = [(batch["record"][0].id, batch) for batch in batches]
        writers = [c for c in trainer.callbacks if hasattr(c, "output_dir")]
        if not args.output and len(writers) != 1:
            raise RuntimeError("expected one Boltz prediction writer (or pass --output)")
        output = args.output or Path(writers[0].output_dir).parent / "benchmark"
        settings = dict(input=arguments[:1], predict_args=getattr(model, "predict_args", None))

        def predict_once(m, batch):
            with torch.inference_mode():
                return m.predict_step(m.transfer_batch_to_device(batch, m.device, 0), 0)

        model.eval()
        compare(model, predict_once, inputs, repeats=args.repeats, output=output, settings=settings)
        print(output / "timings.json")
        adapters.install(model)  # the structures on disk come from the optimized recipe
        try:
            return original_predict(trainer, model, *positional, **keywords)
        finally:
            adapters.uninstall(model)

    Trainer.predict = predict
    try:
        return cli(["predict", *arguments, "--no_kernels"], standalone_mode=False)
    finally:
        Trainer.predict = original_predict


if __name__ == "__main__":
    main()
