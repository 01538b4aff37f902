"""CLI `chat` (one user turn per input line, the conversation kept as context, /reset and
/exit) and `ls` (models in the local store, with digest verification) on CPU."""
import json

from syntropy_b200.cli.main import main


def test_chat_turns_from_a_file(tmp_path, capsys):
    f = tmp_path / "turns.txt"
    f.write_text("hello there\n/reset\nsecond turn\n\n/exit\nnot read\n")
    main(["-o", "model.name=tiny-llama", "-o", "model.max_seq_len=256", "-o", "sched.max_batch=2", "chat",
          "--device", "cpu", "--input", str(f), "--max-tokens", "4", "--temperature", "0", "--json"])
    lines = [json.loads(x) for x in capsys.readouterr().out.strip().splitlines()]
    assert len(lines) == 2 and all(d["tokens"] <= 4 and isinstance(d["reply"], str) for d in lines)


def test_ls_lists_and_verifies_store(tmp_path, capsys):
    from syntropy_b200.store.local import ModelStore
    src = tmp_path / "m"
    src.mkdir()
    (src / "config.json").write_text("{}")
    (src / "w.bin").write_bytes(b"\x01" * 100)
    st = ModelStore(str(tmp_path / "store"))
    st.add("tiny", str(src))
    main(["ls", "--store", str(tmp_path / "store"), "--verify"])
    d = json.loads(capsys.readouterr().out.strip())
    assert d["name"] == "tiny" and d["files"] == 2 and d["bytes"] == 102 and d["damaged"] == []
    (tmp_path / "store" / "tiny" / "w.bin").write_bytes(b"\x02" * 100)
    main(["ls", "--store", str(tmp_path / "store"), "--verify"])
    assert json.loads(capsys.readouterr().out.strip())["damaged"] == ["w.bin"]
