"""Dense decoder-only GPT built on the fused sm_100a layer functions."""

from .builder import BuiltGPTPipeline, BuiltGPTStage, GPTModelBuilder, GPTPipeline, GPTPipelineStage
from .factory import DenseGPTComponents, GPTComponentFactory
from .model import GPTAttention, GPTLayer, GPTMLP, GPTModel, GPTOutput
from .tied_embeddings import TiedEmbeddingSynchronizer
from nano_megatron_b200.pipeline_parallel.partition import LayerPartition

__all__ = [n for n in dir() if not n.startswith("_")]
