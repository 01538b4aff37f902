"""Prefix cache: chained page hashes, sharing and eviction; engine outputs identical with
and without the cache while later requests reuse earlier requests' pages."""
import torch

from syntropy_b200.kv.paged import BlockAllocator
from syntropy_b200.kv.prefix import PrefixCache
from syntropy_b200.models.config import get_config
from syntropy_b200.models.transformer import prepare_weights
from syntropy_b200.runtime.engine import LLMEngine, SamplingParams
from syntropy_b200.runtime.runner import ModelRunner


def test_prefix_cache_match_insert_evict():
    a = BlockAllocator(10)
    pc = PrefixCache(a, block_size=4)
    toks = list(range(13))
    blocks = [a.alloc() for _ in range(4)]
    pc.insert(toks, blocks)
    assert pc.size == 3
    got, n = pc.match(toks[:9] + [99, 98, 97])
    assert got == blocks[:2] and n == 8
    got2, n2 = pc.match([7] + toks[1:12])
    assert got2 == [] and n2 == 0
    for b in got:
        a.free(b)
    for b in blocks:
        a.free(b)
    assert pc.evict(10) == 3 and a.num_free == 9


def test_engine_prefix_reuse_same_tokens():
    cfg = get_config("tiny-qwen-moe")
    mw = prepare_weights(cfg, "cpu", seed=2)
    g = torch.Generator().manual_seed(0)
    base = torch.randint(0, cfg.vocab, (40,), generator=g).tolist()
    prompts = [base + [1, 2, 3], base + [4, 5], base[:33]]
    want = [LLMEngine(ModelRunner(mw, max_batch=4, max_seq_len=128)).generate([p], SamplingParams(max_tokens=5))[0]
            for p in prompts]
    eng = LLMEngine(ModelRunner(mw, max_batch=4, max_seq_len=128), prefix_cache=True)
    got = [eng.generate([p], SamplingParams(max_tokens=5))[0] for p in prompts]
    assert got == want
    assert eng.prefix.hits >= 2
    assert eng.finished[1].cached_tokens == 32
