"""Loss curve on one B200 against the reference implementation (when it is installed).

Both frameworks train the same model from the same seed on the same synthetic batches in
bf16: ours through its sm_100a kernels, the reference through its own PyTorch code path
(the same construction as the benchmark's reference arm). Initial weights are identical
(the same ParallelRNG initialisation, checked bit for bit on CPU), so the per-step losses
must agree within bf16 tolerance. Each framework runs in its own child process.
"""

import json
import os
import subprocess
import sys
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).parents[1]
REF = ROOT / "baseline" / "_ref"

_CONFIG = {
    "distributed": {"backend": "nccl", "device": "cuda", "timeout_minutes": 5},
    "parallel": {"tensor": 1, "pipeline": 1, "context": 1, "expert": 1, "data": 1},
    "model": {"layers": 4, "hidden_size": 1024, "ffn_hidden_size": 2736, "heads": 16,
              "kv_heads": 16, "seq_length": 512, "vocab_size": 8192, "dropout": 0.0,
              "tie_embeddings": True},
    "precision": {"params": "bfloat16", "compute": "bfloat16", "grad_reduce": "float32"},
    "optimizer": {"lr": 5e-4, "betas": [0.9, 0.95], "eps": 1e-8, "weight_decay": 0.1,
                  "clip_grad_norm": 1.0},
    "lr_scheduler": {"schedule": "cosine", "warmup_steps": 0, "decay_steps": 100,
                     "min_lr": 5e-5},
    "training": {"micro_batch_size": 4, "gradient_accumulation_steps": 2, "max_steps": 100,
                 "seed": 1234, "log_interval": 1},
    "wandb": {"enabled": False},
}
STEPS = 8

_RUNNER = r'''
import json, sys
import torch
impl, cfg_json, steps = sys.argv[1], sys.argv[2], int(sys.argv[3])
d = json.loads(cfg_json)
if impl == "ours":
    from nano_megatron_b200.config import config_from_dict
    from nano_megatron_b200.distributed import DistributedRuntime
    from nano_megatron_b200.training import Trainer
    from nano_megatron_b200.training.engine import build_training_components
    d["kernels"] = {"backend": "b200"}
    cfg = config_from_dict(d)
    runtime = DistributedRuntime(cfg.distributed).initialize()
    comps = build_training_components(cfg, runtime)
    trainer = Trainer(config=cfg, model=comps.model, parallel=comps.parallel,
                      data_parallel=comps.data_parallel, rng=comps.rng, device=runtime.device)
else:
    from nano_megatron.config import config_from_dict
    from nano_megatron.data_parallel import build_data_parallel_strategy
    from nano_megatron.distributed import DistributedRuntime
    from nano_megatron.models.gpt import DenseGPTComponents, GPTModelBuilder
    from nano_megatron.nn.kernels import build_kernel_backend
    from nano_megatron.context_parallel import build_context_parallel_attention
    from nano_megatron.parallel import (ParallelContext, ParallelRNG, ParameterDomainRegistry,
                                        RNGStream)
    from nano_megatron.training import Trainer
    cfg = config_from_dict(d)
    runtime = DistributedRuntime(cfg.distributed).initialize()
    parallel = ParallelContext.create(runtime, cfg.parallel)
    rng = ParallelRNG.from_context(cfg.training.seed, parallel)
    torch.manual_seed(rng.seed(RNGStream.DENSE_INIT))
    kernels = build_kernel_backend(cfg.kernels, parallel)
    builder = GPTModelBuilder(
        DenseGPTComponents(cp_attention=build_context_parallel_attention(cfg.context_parallel,
                                                                         parallel)),
        parameter_domains=ParameterDomainRegistry(),
        activation_checkpoint_config=cfg.activation_checkpoint)
    built = builder.build_stage(cfg.model, parallel, kernels, rng=rng)
    model = built.model.to(device=runtime.device, dtype=torch.bfloat16)
    strategy = build_data_parallel_strategy(cfg.data_parallel, cfg.offload, parallel,
                                            built.parameter_domains)
    trainer = Trainer(config=cfg, model=model, parallel=parallel, data_parallel=strategy,
                      rng=rng)
g = torch.Generator().manual_seed(77)
losses = []
S = d["model"]["seq_length"]
for _ in range(steps):
    # learnable data: each next token is a fixed function of the current one
    ids = torch.empty(8, S + 1, dtype=torch.long)
    ids[:, 0] = torch.randint(0, 512, (8,), generator=g)
    for i in range(S):
        ids[:, i + 1] = (ids[:, i] * 3 + 1) % 512
    out = trainer.train_step({"input_ids": ids[:, :-1], "labels": ids[:, 1:]})
    if isinstance(out, dict):
        losses.append(float(out["loss_sum"]) / float(out["token_count"]))
    else:   # the reference returns a StepOutput whose metrics hold the token-mean loss
        losses.append(float(out.metrics["loss"]))
print("LOSSES " + json.dumps(losses))
'''


def _run(impl: str) -> list:
    env = dict(os.environ)
    env["PYTHONPATH"] = os.pathsep.join([str(REF if impl == "reference" else ROOT),
                                         env.get("PYTHONPATH", "")])
    r = subprocess.run([sys.executable, "-c", _RUNNER, impl, json.dumps(_CONFIG), str(STEPS)],
                       env=env, capture_output=True, text=True, timeout=900, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-4000:]
    line = [x for x in r.stdout.splitlines() if x.startswith("LOSSES ")][-1]
    return json.loads(line[len("LOSSES "):])


def test_bf16_loss_curve_matches_reference():
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    if not (REF / "nano_megatron").is_dir():
        pytest.skip("reference implementation not installed")
    ours, theirs = _run("ours"), _run("reference")
    assert len(ours) == len(theirs) == STEPS
    out = os.environ.get("NMB_PARITY_OUT")
    if out:   # keep the two curves for the record (a summary is committed under profiles/)
        with open(out, "w") as f:
            json.dump({"ours": ours, "reference": theirs,
                       "max_rel_diff": max(abs(a - b) / abs(b) for a, b in zip(ours, theirs))},
                      f)
    # identical initial weights and data: the first loss agrees to bf16 rounding, later
    # steps within bf16 training noise (the reference updates bf16 parameters in place,
    # this framework keeps fp32 masters). Measured on B200 over these 8 steps: at most
    # 0.17 % apart, so 1 % leaves a 6x margin.
    assert ours[0] == pytest.approx(theirs[0], rel=5e-3), (ours, theirs)
    for a, b in zip(ours, theirs):
        assert a == pytest.approx(b, rel=1e-2), (ours, theirs)
    assert ours[-1] < ours[0] - 0.3 and theirs[-1] < theirs[0] - 0.3, (ours, theirs)
