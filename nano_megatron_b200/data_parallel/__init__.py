"""Data parallelism: DDP and ZeRO-1/2/3 over flat fp32 gradient buffers."""

from .buffers import Bucket, FlatBuffers, ParamSlice, unique_named_parameters
from .offload import ActivationOffloader, OffloadPolicy, OptimizerStateStorage
from .strategies import (
    DataParallelStrategy,
    DDPStrategy,
    FlatShardZeROStrategy,
    ReplicatedStrategy,
    Zero1Strategy,
    Zero2Strategy,
)
from .zero3 import Zero3Strategy

# the reference's spellings of the ZeRO strategy classes and of a bucket's parameter
# range (same fields; this one also records whether the gradient is SP-replicated)
ZeRO1Strategy, ZeRO2Strategy, ZeRO3Strategy = Zero1Strategy, Zero2Strategy, Zero3Strategy
ParameterSlice = ParamSlice

_STRATEGIES = {"ddp": DDPStrategy, "replicated": ReplicatedStrategy, "zero1": Zero1Strategy,
               "zero2": Zero2Strategy, "zero3": Zero3Strategy}


def build_data_parallel_strategy(config, offload, parallel, parameter_domains):
    mode = str(getattr(getattr(config, "mode", "ddp"), "value", getattr(config, "mode", "ddp")))
    mode = mode.lower().replace("-", "")
    if mode not in _STRATEGIES:
        raise ValueError(f"unknown data-parallel mode {mode!r}; choose one of "
                         f"{', '.join(sorted(_STRATEGIES))}")
    return _STRATEGIES[mode](config=config, offload=offload, parallel=parallel,
                             parameter_domains=parameter_domains)


__all__ = [n for n in dir() if not n.startswith("_")]
