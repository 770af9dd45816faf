"""End-to-end CLI flows on CPU: tokenizer tools, train -> resume -> export -> generate.

Reference counterparts: tests/integration/test_cli_train.py, test_cli_tokenizer.py,
test_cli_export_generate.py.
"""

from __future__ import annotations

import json
from pathlib import Path

import pytest

DEMO = Path(__file__).parents[1] / "examples" / "data" / "tokenizer_demo.jsonl"


def _json_out(capsys) -> dict:
    return json.loads(capsys.readouterr().out.strip().splitlines()[-1])


def test_tokenizer_cli(tmp_path, capsys):
    from nano_megatron_b200.cli import tokenizer as cli

    cli.main(["train", "--input", str(DEMO), "--output", str(tmp_path / "tok"),
              "--vocab-size", "300", "--min-frequency", "1"])
    r = _json_out(capsys)
    assert r["documents"] == 12 and r["vocab_size"] <= 300
    cli.main(["split", "--input", str(DEMO), "--train-output", str(tmp_path / "tr.jsonl"),
              "--validation-output", str(tmp_path / "va.jsonl"), "--validation-fraction", "0.3"])
    s = _json_out(capsys)
    assert s["train_documents"] + s["validation_documents"] == 12
    cli.main(["preprocess", "--input", str(DEMO), "--output", str(tmp_path / "c.pt"),
              "--tokenizer", str(tmp_path / "tok")])
    pt = _json_out(capsys)
    cli.main(["preprocess", "--input", str(DEMO), "--output", str(tmp_path / "c.mmap"),
              "--tokenizer", str(tmp_path / "tok"), "--format", "mmap"])
    mm = _json_out(capsys)
    assert pt["corpus_fingerprint"] == mm["corpus_fingerprint"] and mm["format"] == "mmap"
    cli.main(["inspect", "--tokenizer", str(tmp_path / "tok"), "--text", "a tiny robot",
              "--add-eos"])
    i = _json_out(capsys)
    assert i["ids"][-1] == i["eos_token_id"] and i["decoded"] == "a tiny robot"
    cli.main(["inspect", "--mmap", str(tmp_path / "c.mmap")])
    assert _json_out(capsys)["documents"] == 12


def _config(tmp_path: Path, vocab: int) -> Path:
    import yaml

    from nano_megatron_b200.config import TrainConfig
    from nano_megatron_b200.config.loader import config_to_dict

    d = config_to_dict(TrainConfig())
    d["distributed"].update(backend="gloo", device="cpu")
    d["model"].update(layers=2, hidden_size=64, ffn_hidden_size=128, heads=4, kv_heads=2,
                      seq_length=16, vocab_size=vocab)
    d["precision"].update(params="float32", compute="float32")
    d["training"].update(micro_batch_size=2, gradient_accumulation_steps=1, max_steps=4,
                         log_interval=1)
    d["optimizer"].update(lr=1e-2)
    d["checkpoint"].update(directory=str(tmp_path / "runs"), save_interval=2, keep_last=3)
    tok = {"path": str(tmp_path / "tok"), "append_eos": True}
    d["data"].update(mmap_path=str(tmp_path / "c.mmap"), tokenizer=tok)
    d["validation"].update(interval=2, batches=1,
                           data={"path": str(tmp_path / "c.pt"), "tokenizer": tok,
                                 "shuffle": False})
    p = tmp_path / "cfg.yaml"
    p.write_text(yaml.safe_dump(d))
    return p


def test_train_resume_export_generate(tmp_path, capsys):
    from nano_megatron_b200.cli import export as ecli
    from nano_megatron_b200.cli import generate as gcli
    from nano_megatron_b200.cli import tokenizer as tcli
    from nano_megatron_b200.cli import train as trcli
    from nano_megatron_b200.training.metric_history import read_metric_history

    tcli.main(["train", "--input", str(DEMO), "--output", str(tmp_path / "tok"),
               "--vocab-size", "300", "--min-frequency", "1"])
    vocab = _json_out(capsys)["vocab_size"]
    for fmt, out in (("pt", "c.pt"), ("mmap", "c.mmap")):
        tcli.main(["preprocess", "--input", str(DEMO), "--output", str(tmp_path / out),
                   "--tokenizer", str(tmp_path / "tok"), "--format", fmt])
    capsys.readouterr()
    cfg = _config(tmp_path, vocab)
    st = trcli.run(cfg, max_steps=2, log=lambda *_: None)
    assert st.step == 2
    run1 = next((tmp_path / "runs").iterdir())
    ck = run1 / "step_00000002"
    assert (ck / ".complete").is_file()
    assert (tmp_path / "runs" / "best_validation.json").exists() or \
        (run1 / "best_validation.json").exists()
    st2 = trcli.run(cfg, resume=ck, max_steps=4, log=lambda *_: None)
    assert st2.step == 4 and st2.consumed_samples == 8
    run2 = sorted((tmp_path / "runs").iterdir())[-1]
    hist = read_metric_history(run2 / "metrics.jsonl")
    assert [r.step for r in hist if r.prefix == "train"] == [1, 2, 3, 4]
    ecli.main(["--checkpoint", str(run2 / "step_00000004"), "--output", str(tmp_path / "art")])
    e = _json_out(capsys)
    assert e["source_step"] == 4 and e["weight_dtype"] == "float32"
    gcli.main(["--model", str(tmp_path / "art"), "--prompt", "a tiny", "--device", "cpu",
               "--max-new-tokens", "5", "--temperature", "0", "--json"])
    g = _json_out(capsys)
    assert len(g["generated_token_ids"]) <= 5 and g["text"].startswith("a tiny")
    with pytest.raises(SystemExit):
        gcli.main(["--model", str(tmp_path / "art")])


def test_train_cli_writes_profiler_trace(tmp_path):
    import yaml

    from nano_megatron_b200.cli import train as trcli
    from nano_megatron_b200.config import TrainConfig
    from nano_megatron_b200.config.loader import config_to_dict

    d = config_to_dict(TrainConfig())
    d["distributed"].update(backend="gloo", device="cpu")
    d["model"].update(layers=1, hidden_size=32, ffn_hidden_size=64, heads=4, seq_length=16,
                      vocab_size=64)
    d["precision"].update(params="float32", compute="float32")
    d["training"].update(micro_batch_size=2, gradient_accumulation_steps=1, max_steps=4)
    d["checkpoint"].update(directory=str(tmp_path / "runs"), save_final=False)
    cfg = tmp_path / "c.yaml"
    cfg.write_text(yaml.safe_dump(d))
    trcli.main(["--config", str(cfg), "--profile-dir", str(tmp_path / "prof"),
                "--profile-steps", "1:3"])
    trace = json.loads((tmp_path / "prof" / "trace_rank0000.json").read_text())
    names = {e.get("name", "") for e in trace.get("traceEvents", [])}
    assert any("step" in n for n in names) or len(names) > 10
