"""Export a training checkpoint as a single-device inference artifact (``nano-megatron-export``)."""

from __future__ import annotations

import argparse
import json
from collections.abc import Sequence
from pathlib import Path
from typing import Any

from nano_megatron_b200.inference import export_checkpoint


def parser() -> argparse.ArgumentParser:
    p = argparse.ArgumentParser(description=__doc__)
    p.add_argument("--checkpoint", type=Path, required=True,
                   help="a finished step_NNNNNNNN directory of a training run (any TP/PP/"
                        "interleaved/ZeRO-3 layout)")
    p.add_argument("--output", type=Path, required=True,
                   help="where to write the artifact; must not exist yet")
    p.add_argument("--config", type=Path,
                   help="YAML to describe the model when the checkpoint's manifest carries no "
                        "readable run config")
    p.add_argument("--tokenizer", type=Path,
                   help="tokenizer artifact to bundle instead of the one the run config names")
    return p


def run_export(checkpoint: Path, output: Path, *, config: Path | None = None,
               tokenizer: Path | None = None) -> dict[str, Any]:
    a = export_checkpoint(checkpoint, output, config_path=config, tokenizer_path=tokenizer)
    src, w = a.manifest["source"], a.manifest["weights"]
    return {"artifact": a.manifest["artifact"], "command": "export",
            "format_version": a.manifest["format_version"], "output": str(output),
            "source_checkpoint": src["checkpoint"], "source_step": src["step"],
            "tokenizer_fingerprint": a.tokenizer.fingerprint,
            "vocab_size": a.model_config.vocab_size, "weight_dtype": w["dtype"],
            "weights_sha256": w["sha256"]}


def main(argv: Sequence[str] | None = None) -> None:
    a = parser().parse_args(argv)
    print(json.dumps(run_export(a.checkpoint, a.output, config=a.config, tokenizer=a.tokenizer),
                     ensure_ascii=False, sort_keys=True))


if __name__ == "__main__":
    main()
