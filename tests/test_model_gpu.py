"""The fused CUDA model (bf16, sm_100a kernels) against the same model on CPU in fp32."""

import pytest
import torch

pytestmark = pytest.mark.gpu

from nano_megatron_b200.config import config_from_dict  # noqa: E402
from nano_megatron_b200.distributed import DistributedRuntime  # noqa: E402
from nano_megatron_b200.training.engine import build_training_components  # noqa: E402


def _build(device: str, **model):
    m = {"layers": 2, "hidden_size": 256, "ffn_hidden_size": 688, "heads": 4, "kv_heads": 4,
         "seq_length": 128, "vocab_size": 1024}
    m.update(model)
    cfg = config_from_dict({"model": m, "distributed": {"device": device,
                                                        "backend": "gloo" if device == "cpu" else "nccl"}})
    rt = DistributedRuntime(cfg.distributed).initialize()
    return build_training_components(cfg, rt)


@pytest.mark.parametrize("model", [dict(), dict(heads=2, kv_heads=1, hidden_size=256),
                                   dict(hidden_size=512, heads=4, kv_heads=2,
                                        ffn_hidden_size=1368),
                                   dict(bias=True)])
def test_cuda_model_matches_cpu_fp32(model):
    torch.manual_seed(0)
    cpu = _build("cpu", **model)
    gpu = _build("cuda", **model)
    ids = torch.randint(0, 1024, (2, 129), generator=torch.Generator().manual_seed(3))
    batch = {"input_ids": ids[:, :-1], "labels": ids[:, 1:]}
    # CPU reference in fp32
    lc = cpu.model(None, batch)
    lc.backward()
    # CUDA model: bf16 params (flattened by the data-parallel strategy)
    strat = gpu.data_parallel
    strat.configure_precision(type("P", (), {"params": "bfloat16", "compute": "bfloat16",
                                             "grad_reduce": "float32"})())
    strat.setup(gpu.model, type("O", (), {"lr": 1e-3, "betas": (0.9, 0.95), "eps": 1e-8,
                                          "weight_decay": 0.0})())
    gb = {k: v.cuda() for k, v in batch.items()}
    lg = gpu.model(None, gb)
    lg.backward()
    torch.cuda.synchronize()
    assert abs(lg.item() - lc.item()) < 2e-2 * abs(lc.item())
    cp = dict(cpu.model.named_parameters())
    for name, p in gpu.model.named_parameters():
        ref = cp[name].main_grad
        got = p.main_grad.float().cpu()
        rel = ((got - ref).norm() / (ref.norm() + 1e-12)).item()
        assert rel < 5e-2, f"{name}: rel grad err {rel}"


def _trainer(graphs: bool):
    from nano_megatron_b200.training import Trainer

    cfg = config_from_dict({
        "model": {"layers": 2, "hidden_size": 256, "ffn_hidden_size": 688, "heads": 4,
                  "kv_heads": 2, "seq_length": 128, "vocab_size": 1024},
        "distributed": {"device": "cuda", "backend": "nccl"},
        "kernels": {"backend": "b200", "cuda_graphs": graphs},
        "training": {"micro_batch_size": 2, "gradient_accumulation_steps": 3, "seed": 11},
        "optimizer": {"lr": 1e-3, "clip_grad_norm": 1.0}})
    rt = DistributedRuntime(cfg.distributed).initialize()
    comps = build_training_components(cfg, rt)
    tr = Trainer(config=cfg, model=comps.model, parallel=comps.parallel,
                 data_parallel=comps.data_parallel, rng=comps.rng)
    return comps, tr


def test_cuda_graph_steps_match_eager_steps():
    """Three optimizer steps replayed from per-microbatch CUDA graphs == eager steps."""
    from nano_megatron_b200.ops._ext import lib

    g = torch.Generator().manual_seed(4)
    batches = [torch.randint(0, 1024, (6, 129), generator=g) for _ in range(3)]
    losses, params = {}, {}
    for graphs in (False, True):
        comps, tr = _trainer(graphs)
        assert tr.schedule.use_graphs == graphs
        ls = []
        for ids in batches:
            out = tr.train_step({"input_ids": ids[:, :-1], "labels": ids[:, 1:]})
            ls.append(float(out["loss_sum"] / out["token_count"]))
        torch.cuda.synchronize()
        losses[graphs] = ls
        params[graphs] = {n: p.detach().float().cpu() for n, p in comps.model.named_parameters()}
        if graphs:
            before = lib().launch_count()
            tr.train_step({"input_ids": batches[0][:, :-1], "labels": batches[0][:, 1:]})
            assert lib().launch_count() - before > 3 * 20  # replays are counted
    for a, b in zip(losses[False], losses[True]):
        assert abs(a - b) < 1e-3 * abs(a), (losses[False], losses[True])
    for n, p in params[False].items():
        rel = ((params[True][n] - p).norm() / (p.norm() + 1e-12)).item()
        assert rel < 1e-3, (n, rel)


def test_fit_raises_on_a_kernel_timeout_status():
    """A status code left by a kernel's bounded wait (set here directly, no kernel times
    out) stops ``fit`` at its next logging step with the decoded reason."""
    from nano_megatron_b200.ops._ext import status_word

    _comps, tr = _trainer(False)

    def batches():
        g = torch.Generator().manual_seed(5)
        while True:
            ids = torch.randint(0, 1024, (6, 129), generator=g)
            yield {"input_ids": ids[:, :-1], "labels": ids[:, 1:]}

    tr.bind_data_iterator(batches())
    word = status_word(torch.device("cuda", torch.cuda.current_device()))
    try:
        word.fill_(0x301)
        with pytest.raises(RuntimeError, match="peer flag wait timed out"):
            tr.fit(max_steps=2, log=None)
    finally:
        word.zero_()
        torch.cuda.synchronize()


def test_forward_is_bitwise_reproducible_and_backward_to_fp32_rounding():
    """Race check: the same step twice from the same state. The forward has no atomics,
    so its loss is bitwise equal; gradients (fp32 atomics in split-K, attention dQ, norm
    and embedding backward) agree to fp32 summation-order rounding."""
    comps, tr = _trainer(False)
    ids = torch.randint(0, 1024, (6, 129), generator=torch.Generator().manual_seed(8))
    micro = tr._prepare_batch({"input_ids": ids[:, :-1], "labels": ids[:, 1:]})
    dp = comps.data_parallel
    runs = []
    for _ in range(2):
        dp.zero_grad()
        acc = tr.schedule.forward_backward(micro)
        dp.finalize_gradients()
        torch.cuda.synchronize()
        runs.append((acc.loss_sum.detach().clone(),
                     {n: p.main_grad.detach().clone() for n, p in comps.model.named_parameters()}))
    (l0, g0), (l1, g1) = runs
    assert torch.equal(l0, l1), (l0, l1)
    for n, a in g0.items():
        b = g1[n]
        assert torch.allclose(a, b, rtol=1e-5, atol=1e-6 * float(a.abs().max())), n
