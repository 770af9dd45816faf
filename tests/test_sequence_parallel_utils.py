"""Sequence-parallel region helpers on two gloo ranks: the sequence scatter (forward keeps
this rank's block, backward all-gathers) and the gradient hooks that sum the gradients of
SP-replicated parameters over the group."""

from __future__ import annotations

import torch

from dist_utils import run_ranks


class _Group:
    def __init__(self, rank, size):
        import torch.distributed as dist

        self.rank, self.size, self.process_group = rank, size, dist.group.WORLD


def _scatter_rank(rank, world):
    from nano_megatron_b200.tensor_parallel import scatter_to_sequence_parallel_region

    g = _Group(rank, world)
    x = torch.arange(24.0).reshape(4, 3, 2).requires_grad_()      # [S, B, H], replicated
    y = scatter_to_sequence_parallel_region(x, g, sequence_dim=0)
    assert torch.equal(y, x.detach()[2 * rank:2 * rank + 2])
    (y * (rank + 1)).sum().backward()
    # backward all-gathers every rank's block gradient: rank r's block is scaled by r + 1
    want = torch.cat([torch.full((2, 3, 2), 1.0), torch.full((2, 3, 2), 2.0)])
    assert torch.equal(x.grad, want)
    z = torch.arange(12.0).reshape(3, 4)
    assert torch.equal(scatter_to_sequence_parallel_region(z, g, sequence_dim=1),
                       z[:, 2 * rank:2 * rank + 2])


def test_sequence_scatter_keeps_the_block_and_gathers_gradients():
    run_ranks(2, _scatter_rank)


def _hook_rank(rank, world):
    from nano_megatron_b200.tensor_parallel import register_sequence_parallel_gradient_hooks

    torch.manual_seed(0)
    norm = torch.nn.LayerNorm(4)                                    # replicated parameters
    g = _Group(rank, world)
    register_sequence_parallel_gradient_hooks(norm, g)
    register_sequence_parallel_gradient_hooks(norm, g)              # idempotent
    full = torch.randn(6, 4, generator=torch.Generator().manual_seed(1))
    norm(full[3 * rank:3 * rank + 3]).pow(2).sum().backward()
    ref = torch.nn.LayerNorm(4)
    ref.load_state_dict(norm.state_dict())
    ref(full).pow(2).sum().backward()                               # the whole sequence
    assert torch.allclose(norm.weight.grad, ref.weight.grad, atol=1e-5)
    assert torch.allclose(norm.bias.grad, ref.bias.grad, atol=1e-5)


def test_gradient_hooks_sum_replicated_parameter_gradients():
    run_ranks(2, _hook_rank)
