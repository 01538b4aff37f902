"""Property-based tests (hypothesis) of the native runtime pieces against Python models: the
4-bit quantiser (native == pure-torch rule, per-element error within half a step), the row <->
tiled layout round trip, the SPSC ring against a deque, the frame codec round trip with CRC
checks, the arena against an interval model, the swap planner against a direct restatement of
its rule, and the JSON automaton against `json.loads`."""
import collections
import json

import pytest
import torch

hypothesis = pytest.importorskip("hypothesis")
from hypothesis import HealthCheck, assume, given, settings  # noqa: E402
from hypothesis import strategies as st  # noqa: E402

from syntropy_b200._ext import ext  # noqa: E402
from syntropy_b200.formats.q4 import dequant_rows_ref, quantize_rows_ref  # noqa: E402

SETTINGS = settings(max_examples=60, deadline=None, derandomize=True, suppress_health_check=[HealthCheck.too_slow])


@SETTINGS
@given(n_tiles=st.integers(1, 3), kg=st.integers(1, 3), scale=st.floats(1e-3, 10.0), seed=st.integers(0, 2**31 - 1))
def test_q4_quantiser_and_layouts(n_tiles, kg, scale, seed):
    N, K = 16 * n_tiles, 64 * kg
    g = torch.Generator().manual_seed(seed)
    w = torch.randn(N, K, generator=g) * scale
    rows = ext().q4_quantize_rows_cpu(w.contiguous())
    assert torch.equal(rows.view(-1), quantize_rows_ref(w).view(-1))
    deq = dequant_rows_ref(rows, N, K)
    d = rows.view(N, K // 32, 20)[..., 0:2].contiguous().view(torch.float16).float()
    step = d.repeat_interleave(32, dim=1).reshape(N, K)
    # |w - deq| <= half a step (+ fp16 rounding of the scale and min)
    assert bool(((w - deq).abs() <= 0.5 * step + 1e-3 * w.abs().amax() + 1e-6).all())
    qw, sm = ext().q4_rows_to_tiled_cpu(rows, N, K)
    # the tiled layout carries the same numbers: the host GEMV over it equals the row product
    x = torch.randn(2, K, generator=g).bfloat16()
    y = ext().cpu_q4t_gemv(qw, sm, x, N, 0)
    ref = x.float() @ deq.t()
    assert torch.allclose(y, ref, rtol=1e-4, atol=1e-4 * (ref.abs().max().item() + 1e-6))


@SETTINGS
@given(ops_=st.lists(st.one_of(st.binary(min_size=0, max_size=24), st.none()), max_size=80))
def test_spsc_ring_matches_deque(ops_):
    ring = ext().SpscRing(8, 24)
    model = collections.deque()
    for op in ops_:
        if op is None:  # pop
            got = ring.pop()
            if model:
                assert got == model.popleft()
            else:
                assert got is None
        else:
            ok = ring.push(op)
            assert ok == (len(model) < 8)
            if ok:
                model.append(op)
        assert ring.size() == len(model)


@SETTINGS
@given(ftype=st.integers(0, 255), flags=st.integers(0, 65535), inst=st.integers(0, 2**62), term=st.integers(0, 2**62),
       seq=st.integers(0, 2**62), step=st.integers(0, 2**62), chan=st.integers(0, 2**62),
       ext_=st.binary(max_size=40), payload=st.binary(max_size=300), flip=st.integers(0, 10**6))
def test_frame_codec_round_trip_and_crc(ftype, flags, inst, term, seq, step, chan, ext_, payload, flip):
    buf = ext().frame_encode(ftype, flags, inst, term, seq, step, chan, ext_, payload)
    rc, spec, e2, p2 = ext().frame_decode(buf)
    # the extension travels zero-padded to a multiple of 64 bytes (the payload starts aligned)
    assert rc == 0 and p2 == payload and e2 == ext_ + bytes(-len(ext_) % 64)
    assert (spec["ftype"], spec["flags"], spec["instance"], spec["epoch_term"], spec["epoch_seq"], spec["step"],
            spec["chan_seq"]) == (ftype, flags, inst, term, seq, step, chan)
    # any single flipped bit is rejected
    b = bytearray(buf)
    bit = flip % (8 * len(b))
    b[bit // 8] ^= 1 << (bit % 8)
    assert ext().frame_decode(bytes(b))[0] != 0


@SETTINGS
@given(reqs=st.lists(st.tuples(st.integers(1, 300), st.sampled_from([1, 16, 64, 256]), st.booleans()), max_size=60))
def test_arena_against_interval_model(reqs):
    cap = 2048
    a = ext().Arena(cap)
    live = {}
    for size, align, release in reqs:
        if release and live:
            off = sorted(live)[len(live) // 2]
            a.release(off)
            del live[off]
            continue
        off = a.alloc(size, align)
        if off < 0:
            continue
        assert off % align == 0 and off + size <= cap
        for o, s in live.items():  # no overlap with a live range
            assert off + size <= o or o + s <= off
        live[off] = size
        assert a.used() == sum(live.values())
    for off in list(live):
        a.release(off)
    assert a.used() == 0 and a.largest_free() == cap


@SETTINGS
@given(scores=st.lists(st.floats(0, 100), min_size=2, max_size=16), data=st.data(),
       max_swaps=st.integers(0, 6), hyst=st.floats(1.0, 2.0))
def test_swap_planner_rule(scores, data, max_swaps, hyst):
    resident = data.draw(st.lists(st.booleans(), min_size=len(scores), max_size=len(scores)))
    plan = ext().tier_plan_swaps(scores, resident, max_swaps, hyst)
    res = list(resident)
    want = []
    for _ in range(max_swaps):
        cold = [e for e in range(len(scores)) if res[e]]
        hot = [e for e in range(len(scores)) if not res[e]]
        if not cold or not hot:
            break
        c = min(cold, key=lambda e: (scores[e], e))
        h = max(hot, key=lambda e: (scores[e], -e))
        if not (scores[h] > hyst * scores[c]) or scores[h] <= 0:
            break
        want.append((c, h))
        res[c], res[h] = False, True
    assert plan == want


_json = st.recursive(st.none() | st.booleans() | st.integers(-10**6, 10**6) |
                     st.floats(allow_nan=False, allow_infinity=False) | st.text(max_size=8),
                     lambda kids: st.lists(kids, max_size=4) | st.dictionaries(st.text(max_size=6), kids, max_size=4),
                     max_leaves=12)


def _json_ok(text: bytes) -> bool:
    trie = ext().TokenTrie([bytes([b]) for b in range(256)])
    c = ext().Constraint.json(trie, -1)
    return all(c.advance(b) for b in text) and c.accepting()


@SETTINGS
@given(obj=st.dictionaries(st.text(max_size=6), _json, max_size=4), indent=st.sampled_from([None, 1]))
def test_json_automaton_accepts_serialised_objects(obj, indent):
    text = json.dumps(obj, indent=indent, ensure_ascii=False).encode()
    # the automaton caps runs of insignificant whitespace at 8 bytes (no runaway indentation)
    assume(max((len(r) for r in __import__("re").findall(rb"[ \n\t\r]+", text)), default=0) <= 8)
    assert _json_ok(text)


@SETTINGS
@given(obj=st.dictionaries(st.text(max_size=4), _json, max_size=3), cut=st.integers(0, 400), byte=st.integers(0, 255))
def test_json_automaton_agrees_with_json_loads(obj, cut, byte):
    text = bytearray(json.dumps(obj, separators=(",", ":")).encode())
    if text:
        text[cut % len(text)] = byte  # a one-byte mutation
    try:
        v = json.loads(bytes(text))
        valid = isinstance(v, dict)
    except (ValueError, UnicodeDecodeError):
        valid = False
    if b"\\" in text and valid:
        return  # json.loads accepts lone surrogate escapes the same way; nothing to compare
    assert _json_ok(bytes(text)) == valid
