"""Format-preserving config writes: one key changes, every other byte of the file stays."""
import pytest

from syntropy_b200.config import load_config
from syntropy_b200.config.write import set_value

TEXT = """# node config
[model]
name = "llama3-8b"   # the preset
max_seq_len = 2048

# scheduling
[sched]
max_batch = 32 # rows
cuda_graphs = true
"""


def test_edit_keeps_comments_and_order(tmp_path):
    p = tmp_path / "c.toml"
    p.write_text(TEXT)
    out = set_value(str(p), "sched.max_batch", "48")
    assert out == TEXT.replace("max_batch = 32 # rows", "max_batch = 48 # rows")
    out = set_value(str(p), "model.name", 'qwen3-235b-a22b "x" # not a comment')
    assert 'name = "qwen3-235b-a22b \\"x\\" # not a comment"   # the preset' in out
    cfg = load_config(str(p), env={})
    assert cfg.sched.max_batch == 48 and cfg.model.name == 'qwen3-235b-a22b "x" # not a comment'
    assert cfg.origin["sched.max_batch"] == f"file {p}:8"


def test_insert_key_and_section(tmp_path):
    p = tmp_path / "c.toml"
    p.write_text(TEXT)
    out = set_value(str(p), "model.seed", "7")
    assert out.splitlines()[4] == "seed = 7" and out.startswith(TEXT.split("\n# scheduling")[0])
    out = set_value(str(p), "tier.kv_budget", "8GiB")
    assert out.endswith('\n[tier]\nkv_budget = "8GiB"\n')
    out = set_value(str(p), "features.disable", "cuda_graph,expert_prefetch")
    assert 'disable = ["cuda_graph", "expert_prefetch"]' in out
    cfg = load_config(str(p), env={})
    assert cfg.model.seed == 7 and cfg.tier.kv_budget == 8 << 30 and cfg.features.disable == ["cuda_graph",
                                                                                               "expert_prefetch"]
    new = tmp_path / "new.toml"
    set_value(str(new), "sched.cuda_graphs", "off")
    assert new.read_text() == "[sched]\ncuda_graphs = false\n"


def test_rejects_bad_keys_and_values(tmp_path):
    p = tmp_path / "c.toml"
    p.write_text(TEXT)
    with pytest.raises(KeyError):
        set_value(str(p), "sched.no_such_key", "1")
    with pytest.raises(ValueError):
        set_value(str(p), "sched.max_batch", "many")
    assert p.read_text() == TEXT  # untouched


def test_cli_config_set_and_get(tmp_path, capsys):
    import json

    from syntropy_b200.cli.main import main
    p = tmp_path / "c.toml"
    p.write_text(TEXT)
    main(["--config", str(p), "config", "set", "sched.max_batch", "40"])
    capsys.readouterr()
    main(["--config", str(p), "config", "get", "sched.max_batch"])
    got = json.loads(capsys.readouterr().out)
    assert got["value"] == 40 and got["origin"] == f"file {p}:8"
