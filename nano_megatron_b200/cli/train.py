"""Train a GPT model from one YAML configuration (``nano-megatron-train``).

Run flow (the reference's, src/nano_megatron/cli/train.py:89-202): load and
validate the config for ``WORLD_SIZE``; load the tokenizer when the data or
validation config names one; build runtime, parallel context, RNG, model and
data-parallel strategy; allocate a timestamped checkpoint run directory on
rank 0 and publish it to every rank; restore ``--resume`` if given (metric
history replayed from the resumed run's ``metrics.jsonl``); bind the
resumable train loader (and validation loader) and ``fit``.
"""

from __future__ import annotations

import argparse
import os
from collections.abc import Sequence
from dataclasses import replace
from datetime import datetime
from pathlib import Path

from nano_megatron_b200.checkpoint import CheckpointManager
from nano_megatron_b200.config import load_config, validate_config
from nano_megatron_b200.data import build_train_dataloader, build_validation_dataloader
from nano_megatron_b200.distributed import DistributedRuntime
from nano_megatron_b200.tokenizer import ByteLevelBPETokenizer, validate_tokenizer_for_model
from nano_megatron_b200.training import Trainer
from nano_megatron_b200.training.engine import build_training_components


def parser() -> argparse.ArgumentParser:
    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    p.add_argument("--config", type=Path, required=True,
                   help="YAML file describing the run (model, parallel layout, data, "
                        "optimizer, ...)")
    p.add_argument("--set", dest="overrides", action="append", default=[], metavar="KEY=VALUE",
                   help="section.field=value applied on top of the YAML; give it once per field")
    p.add_argument("--resume", type=Path,
                   help="step directory of an earlier run to continue from (weights, "
                        "optimizer, data position, RNG)")
    p.add_argument("--max-steps", type=int,
                   help="stop at this step in this invocation, without changing the stored "
                        "config")
    p.add_argument("--profile-dir", type=Path,
                   help="write a torch.profiler Chrome trace per rank for --profile-steps")
    p.add_argument("--profile-steps", default="2:4", metavar="START:STOP",
                   help="completed-step window to profile (default 2:4)")
    return p


def run_timestamp() -> str:
    return datetime.now().astimezone().strftime("%Y%m%d-%H%M%S-%f")


def allocate_run_directory(base: Path, runtime) -> Path:
    """Rank 0 creates ``<base>/<timestamp>[-NN]``; every rank receives the same path."""
    local = None
    if runtime.is_primary:
        try:
            base.mkdir(parents=True, exist_ok=True)
            stamp = run_timestamp()
            cand, n = base / stamp, 0
            while True:
                try:
                    cand.mkdir(parents=False, exist_ok=False)
                    break
                except FileExistsError:
                    n += 1
                    cand = base / f"{stamp}-{n:02d}"
            local = (str(cand), None)
        except BaseException as e:  # noqa: BLE001
            local = (None, f"{type(e).__name__}: {e}")
    got = runtime.all_gather_object(local)[0]
    if not isinstance(got, tuple) or len(got) != 2:
        raise RuntimeError("rank 0 returned an invalid checkpoint directory result")
    d, err = got
    if err is not None:
        raise RuntimeError(f"failed to allocate checkpoint run directory: {err}")
    if not isinstance(d, str) or not d:
        raise RuntimeError("rank 0 returned an empty checkpoint run directory")
    return Path(d)


def load_run_tokenizer(config):
    tc = config.data.tokenizer
    if tc is None and config.validation.data is not None:
        tc = config.validation.data.tokenizer
    if tc is None:
        return None
    tok = ByteLevelBPETokenizer.load(tc.path)
    validate_tokenizer_for_model(tok, config.model)
    return tok


def run(config_path: Path, *, overrides: Sequence[str] = (), resume: Path | None = None,
        max_steps: int | None = None, log=print, profile_dir: Path | None = None,
        profile_steps: str = "2:4"):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    config = load_config(config_path, overrides=overrides, world_size=world)
    validate_config(config, world_size=world)
    tokenizer = load_run_tokenizer(config)
    with DistributedRuntime(config.distributed) as runtime:
        runtime.initialize()
        comps = build_training_components(config, runtime)
        run_dir = allocate_run_directory(Path(config.checkpoint.directory), runtime)
        config = replace(config, checkpoint=replace(config.checkpoint, directory=run_dir))
        if runtime.is_primary:
            log(f"checkpoint run directory: {run_dir}")
        ckpt = CheckpointManager(config=config.checkpoint, parallel=comps.parallel,
                                 run_config=config)
        from nano_megatron_b200.distributed.health import PeerHealth

        health = PeerHealth.from_default_group() if runtime.world_size > 1 else None
        if health is not None:
            health.start()
        trainer = Trainer(config=config, model=comps.model, parallel=comps.parallel,
                          data_parallel=comps.data_parallel, checkpoint=ckpt, rng=comps.rng,
                          health=health, metrics_path=run_dir / "metrics.jsonl",
                          resume_metrics_path=None if resume is None
                          else Path(resume).parent / "metrics.jsonl")
        if profile_dir is not None:
            from nano_megatron_b200.utils.profiling import StepProfiler

            a, b = (int(x) for x in profile_steps.split(":"))
            trainer.profiler = StepProfiler(profile_dir, a, b, rank=runtime.rank)
        try:
            if resume is not None:
                trainer.load_checkpoint(resume)
            data = build_train_dataloader(config, comps.parallel, tokenizer=tokenizer,
                                          max_steps=max_steps)
            if trainer.batch_router.is_source:
                fp = getattr(data, "data_fingerprint", None)
                if not isinstance(fp, str):
                    raise TypeError("source data loader must expose data_fingerprint")
                trainer.bind_data_iterator(data, data_fingerprint=fp)
            else:
                trainer.data_iterator = iter(data)
            if config.validation.interval > 0:
                trainer.bind_validation_data(build_validation_dataloader(
                    config, comps.parallel, tokenizer=tokenizer))
            primary = runtime.is_primary
            state = trainer.fit(max_steps=max_steps, log=log)
        finally:
            if trainer.profiler is not None:
                trainer.profiler.close()
            trainer.close()
            ckpt.close()
            if health is not None:
                health.stop()
            comps.close(trainer)    # graphs, peer memory, subgroups, default group, in order
        if primary:
            log(f"finished step={state.step} samples={state.consumed_samples} "
                f"tokens={state.consumed_tokens}")
        return state


def main(argv: Sequence[str] | None = None) -> None:
    a = parser().parse_args(argv)
    run(a.config, overrides=a.overrides, resume=a.resume, max_steps=a.max_steps,
        profile_dir=a.profile_dir, profile_steps=a.profile_steps)


if __name__ == "__main__":
    main()
