"""Grammar-constrained decoding: the native JSON automaton accepts exactly RFC 8259 texts with an
object at the top level; token masks from the vocabulary trie equal a brute-force check of every
token; an engine run on CPU under a constraint produces valid JSON / one of the choices."""
import json
import random

import pytest
import torch

from syntropy_b200._ext import ext
from syntropy_b200.text.constrain import allowed, make_constraint, vocab_bytes


def _byte_trie():
    vb = [bytes([b]) for b in range(256)]
    return ext().TokenTrie(vb), vb


def _accepts(text: bytes) -> bool:
    trie, _ = _byte_trie()
    c = make_constraint(trie, None, {"type": "json"})
    return all(c.advance(b) for b in text) and c.accepting()


@pytest.mark.parametrize("text", [b'{}', b' {"a": 1}', b'{"a": [1, 2.5e-3, -0, true, false, null, "x\\u00e9\\n"]}',
                                  b'{"k": {"n": {}}, "l": [[], [{}]]}', b'{"s": "\xc3\xa9"}'])
def test_json_accepts_valid(text):
    assert _accepts(text)
    json.loads(text)


@pytest.mark.parametrize("text", [b'[]', b'{"a" 1}', b'{"a": 01}', b'{"a": tru}', b'{"a": 1,}', b'{"a": "\x01"}',
                                  b'{"a": 1}}', b'{"a": 1.}', b'{a: 1}', b'{"a": 1]', b'{"a": "\xc3("}',
                                  b'{"a": "\xed\xa0\x80"}', b'{"a": "\xff"}'])
def test_json_rejects_invalid(text):
    assert not _accepts(text)


def test_masks_match_brute_force():
    rnd = random.Random(0)
    alphabet = list(b'{}[]",:0123456789-.eE+ truefalsnl\\abcxyz\n')
    vocab = [bytes([b]) for b in range(256)] + [b""] * 3
    for _ in range(400):
        vocab.append(bytes(rnd.choice(alphabet) for _ in range(rnd.randint(2, 6))))
    vocab += [b'{"', b'": ', b'", "', b'"}', b'}}', b']}', b'true', b'null,']
    trie = ext().TokenTrie(vocab)
    eos = 256
    for prefix in (b'', b'{', b'{"ab', b'{"a": ', b'{"a": [1', b'{"a": [1, -', b'{"a": {"b": "c"', b'{"a": 1}'):
        c = make_constraint(trie, eos, {"type": "json"})
        assert all(c.advance(b) for b in prefix)
        got = allowed(c.mask(), len(vocab))
        for i, tb in enumerate(vocab):
            if i == eos:
                want = c.accepting()
            elif not tb:
                want = False
            else:
                probe = make_constraint(trie, eos, {"type": "json"})
                want = all(probe.advance(b) for b in prefix + tb)
            assert bool(got[i]) == want, (prefix, tb)


def test_choices_constraint():
    trie, _ = _byte_trie()
    c = make_constraint(trie, None, {"choices": ["yes", "no", "maybe"]})
    m = allowed(c.mask(), 256)
    assert sorted(torch.nonzero(m).flatten().tolist()) == sorted(b"ynm")
    assert c.advance(ord("n")) and not c.advance(ord("x")) and c.advance(ord("o")) and c.finished()


def test_engine_constrained_generation_cpu():
    from syntropy_b200.models.config import get_config
    from syntropy_b200.models.transformer import prepare_weights
    from syntropy_b200.runtime.engine import LLMEngine, SamplingParams
    from syntropy_b200.runtime.runner import ModelRunner
    from syntropy_b200.text.tokenizer import ByteTokenizer
    cfg = get_config("tiny-llama")
    mw = prepare_weights(cfg, torch.device("cpu"), seed=0)
    eng = LLMEngine(ModelRunner(mw, max_batch=4, max_seq_len=256), eos_token_id=ByteTokenizer.EOS)
    eng.set_tokenizer(ByteTokenizer(cfg.vocab))
    tok = ByteTokenizer(cfg.vocab)
    outs = eng.generate([tok.encode("pick:"), tok.encode("json:")],
                        [SamplingParams(max_tokens=12, constraint={"choices": ["alpha", "beta"]}),
                         SamplingParams(max_tokens=200, temperature=0.8, seed=3, constraint={"type": "json"})])
    assert tok.decode(outs[0]) in ("alpha", "beta")
    ids = [t for t in outs[1] if t != ByteTokenizer.EOS]
    c = make_constraint(eng._token_trie(), None, {"type": "json"})
    assert all(c.advance(t) for t in ids)  # never leaves the grammar
    if len(outs[1]) < 200:  # finished by the grammar, not by length
        assert c.finished()
        json.loads(bytes(t - ByteTokenizer.OFFSET for t in ids))
