"""Config layering: typed values (sizes, durations), file:line origins in errors, validation
of the kernels / spec / tier sections, and the CLI engine honouring the spec section."""
import pytest

from syntropy_b200.config.schema import load_config, parse_duration, parse_size


def test_typed_values():
    assert parse_size("64GiB") == 64 << 30 and parse_size("512 MB") == 512 * 10**6 and parse_size(4096) == 4096
    assert parse_duration("250ms") == 0.25 and parse_duration("1m") == 60.0 and parse_duration(2) == 2.0
    with pytest.raises(ValueError):
        parse_size("12 parsecs")
    cfg = load_config(env={}, overrides=["tier.kv_budget=2GiB", "kernels.spin_timeout=500ms"])
    assert cfg.tier.kv_budget == 2 << 30 and cfg.kernels.spin_timeout == 0.5


def test_file_line_origin_in_errors(tmp_path):
    p = tmp_path / "node.toml"
    p.write_text("[model]\nname = 'small-llama'\n\n[tier]\n# cache\nexpert_cache_frac = 1.5\n")
    with pytest.raises(ValueError, match=r"tier.expert_cache_frac must be in \[0, 1\] \(file .*node.toml:6\)"):
        load_config(str(p), env={})
    p.write_text("[kernels]\nspin_timeout = 'soon'\n")
    with pytest.raises(ValueError, match=r"kernels.spin_timeout: not a duration.*node.toml:2"):
        load_config(str(p), env={})


def test_section_validation_and_precedence(tmp_path):
    p = tmp_path / "n.toml"
    p.write_text("[spec]\ndrafter = 'ngram'\ngamma = 3\n")
    cfg = load_config(str(p), env={"SYN_SPEC_GAMMA": "4"}, overrides=[])
    assert cfg.spec.gamma == 4 and cfg.origin["spec.gamma"] == "env SYN_SPEC_GAMMA"
    with pytest.raises(ValueError, match="spec.draft_model is required"):
        load_config(env={}, overrides=["spec.drafter=draft"])
    with pytest.raises(ValueError, match="spec.drafter must be one of"):
        load_config(env={}, overrides=["spec.drafter=oracle"])


def test_cli_engine_spec_section():
    from syntropy_b200.cli.main import _engine_from_config
    from syntropy_b200.runtime.engine import SamplingParams
    from syntropy_b200.runtime.spec import DraftModelDrafter, NgramDrafter
    base = ["model.name=tiny-llama", "model.max_seq_len=96", "sched.max_batch=4"]
    eng, _ = _engine_from_config(load_config(env={}, overrides=base), "cpu")
    want = eng.generate([[3, 4, 5, 6]], SamplingParams(max_tokens=10))
    eng, _ = _engine_from_config(load_config(env={}, overrides=base + ["spec.drafter=ngram", "spec.gamma=3"]), "cpu")
    assert isinstance(eng.spec.drafter, NgramDrafter) and eng.spec.gamma == 3
    assert eng.generate([[3, 4, 5, 6]], SamplingParams(max_tokens=10)) == want
    eng, _ = _engine_from_config(load_config(env={}, overrides=base + ["spec.drafter=draft",
                                                                         "spec.draft_model=tiny-llama"]), "cpu")
    assert isinstance(eng.spec.drafter, DraftModelDrafter)
    assert eng.generate([[3, 4, 5, 6]], SamplingParams(max_tokens=10)) == want
    assert eng.acceptance_rate > 0.9  # the same model drafts for itself


def test_feature_kill_switches():
    """features.disable names switches from a closed set (a typo is an error, not a no-op);
    disabling `speculative` serves without drafts even when spec.drafter asks for them."""
    from syntropy_b200.cli.main import _engine_from_config
    with pytest.raises(ValueError, match="unknown switches"):
        load_config(env={}, overrides=["features.disable=cuda_graphs"])
    base = ["model.name=tiny-llama", "model.max_seq_len=96", "sched.max_batch=4", "spec.drafter=ngram"]
    cfg = load_config(env={}, overrides=base + ["features.disable=speculative,cuda_graph"])
    assert not cfg.feature("speculative") and not cfg.feature("cuda_graph") and cfg.feature("cpu_tier")
    eng, _ = _engine_from_config(cfg, "cpu")
    assert eng.spec is None and not eng.runner.use_graphs
