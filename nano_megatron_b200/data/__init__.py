"""Token corpora, fixed-length datasets and the resumable native batch loader."""

from .corpus import TokenCorpus, build_token_corpus, iter_jsonl_text, preprocess_jsonl
from .datasets import (
    FixedLengthTokenDataset,
    MMapTokenDataset,
    RandomTokenDataset,
    build_train_dataset,
)
from .loader import StatefulDataLoader, build_train_dataloader, build_validation_dataloader
from .mmap_corpus import (
    MMapCorpusError,
    MMapTokenCorpus,
    preprocess_jsonl_mmap,
    preprocess_texts_mmap,
)
from .tinystories import (
    TINYSTORIES_EMPTY_RECORDS,
    TINYSTORIES_SAMPLE_SEED,
    TINYSTORIES_SAMPLE_STORIES,
    TINYSTORIES_TRAIN_RECORDS,
    TINYSTORIES_TRAIN_STORIES,
    TINYSTORIES_VALIDATION_STORIES,
    prepare_tinystories_500k,
)
from .tinystories_corpus import (
    TinyStoriesCorpusError,
    build_tinystories_corpus,
    prepare_tinystories_corpus,
    validate_tinystories_corpus,
)

__all__ = [n for n in dir() if not n.startswith("_")]
