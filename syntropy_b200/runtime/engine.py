"""LLM engine: request intake, continuous batching, prefill/decode steps, sampling state.

Scheduling (reference design: plan/rfcs/RFC-0012-execution-scheduler.md): FCFS admission
while KV pages last; a step is either a prefill batch (whole prompts up to a token budget)
or one decode step over every running sequence.  Each sequence carries its sampling key
(seed, stream) and ``rng_counter`` (plan/decisions/ADR-0107-counter-based-sampling-rng.md).
"""
from __future__ import annotations

import itertools
import random
import time
from collections import deque
from dataclasses import dataclass, field

import torch

from .._ext import ext

from .. import ops
from .runner import ModelRunner


MAX_LOGPROBS = 20  # most alternatives per token a request may ask for


@dataclass
class SamplingParams:
    max_tokens: int = 16
    temperature: float = 0.0
    top_k: int = 0
    top_p: float = 1.0
    seed: int | None = None
    stop_token_ids: tuple = ()
    ignore_eos: bool = True
    constraint: object = None  # {"type": "json"} or {"choices": [...]} (text/constrain.py)
    repetition_penalty: float = 1.0  # > 1 discourages every token of the prompt and output
    frequency_penalty: float = 0.0   # subtracted once per earlier occurrence in the output
    presence_penalty: float = 0.0    # subtracted once if the token occurred in the output
    logit_bias: dict | None = None   # {token id: added logit}
    logprobs: int | None = None      # record each emitted token's log-probability under the model's
    #                                  own distribution and the `logprobs` most likely alternatives

    @property
    def processed(self) -> bool:
        """Whether logits need processing before the draw (penalties or bias)."""
        return (self.repetition_penalty != 1.0 or self.frequency_penalty != 0.0 or self.presence_penalty != 0.0
                or bool(self.logit_bias))


@dataclass
class Sequence:
    seq_id: int
    prompt: list
    params: SamplingParams
    output: list = field(default_factory=list)
    logprobs: list = field(default_factory=list)  # per emitted token, when params.logprobs is set
    blocks: list = field(default_factory=list)
    status: str = "waiting"  # waiting | running | finished
    cached_tokens: int = 0   # prompt tokens served from the prefix cache
    prefilled: int = 0       # prompt tokens whose K/V are written (chunked prefill)
    mtp_draft: list | None = None
    finish_reason: str | None = None
    seed: int = 0
    stream: int = 0
    rng_counter: int = 0
    t_arrival: float = 0.0
    t_first_token: float | None = None
    constraint: object = None  # native automaton state of a constrained request
    t_finished: float | None = None

    @property
    def n_tokens(self) -> int:
        return len(self.prompt) + len(self.output)


@dataclass
class StepOutput:
    seq_id: int
    new_tokens: list
    finished: bool
    finish_reason: str | None = None
    logprobs: list | None = None  # records of new_tokens, when the request asked for them


class LLMEngine:
    def __init__(self, runner: ModelRunner, max_prefill_tokens: int = 8192, eos_token_id: int | None = None,
                 dist_ctx=None, prefix_cache: bool = False, spec=None, rebalance_every: int = 64,
                 chunk_tokens: int | None = None, kv_host_bytes: int | None = None,
                 kv_spill_dir: str | None = None):
        self.runner = runner
        # Chunked prefill (reference plan/rfcs/RFC-0012-execution-scheduler.md:299-314): prompts
        # enter the KV cache at most `chunk_tokens` tokens per step, and every step first runs
        # the decode rows of the running sequences, so a long prompt delays them by one chunk at
        # most.  None: whole prompts (up to max_prefill_tokens per step), prefill steps alone.
        if chunk_tokens is not None and (chunk_tokens < 1 or spec is not None or runner.pp is not None or
                                         (dist_ctx is not None and dist_ctx.enabled)):
            raise ValueError("chunk_tokens: a positive count, without speculation, pipeline stages or lockstep ranks")
        self.chunk_tokens = chunk_tokens
        self.prefilling: list[Sequence] = []  # admitted, prompt partly in the KV cache (chunked prefill)
        self.step_log: list | None = None     # when a list: (decode rows, prefill tokens) per step
        self.rebalance_every = rebalance_every  # decode steps between expert-cache adaptations (0: never)
        self.spec = spec  # runtime.spec.SpecConfig or None
        self.prefix = None
        if prefix_cache:
            from ..kv.prefix import PrefixCache
            self.prefix = PrefixCache(runner.kv.alloc, runner.kv.block_size)
        # Under expert parallelism every rank must take the same kind of step (the MoE
        # layers exchange rows), so step kinds are agreed over the host control group.
        self.dist = dist_ctx if (dist_ctx is not None and dist_ctx.enabled) else None
        self.cfg = runner.cfg
        self.max_prefill_tokens = max_prefill_tokens
        self.eos = eos_token_id
        self.waiting: deque[Sequence] = deque()
        self.running: list[Sequence] = []
        # preempted sequences whose KV pages wait below VRAM: (sequence, SwapStore entry); the
        # store keeps them in host RAM up to kv_host_bytes, then in pack files under kv_spill_dir
        from ..kv.tiers import SwapStore
        self.swapped: deque = deque()
        self.kv_store = SwapStore(kv_host_bytes, kv_spill_dir)
        self.finished: dict[int, Sequence] = {}
        self._ids = itertools.count()
        self._boot_seed = random.getrandbits(63)
        self.stats = {"prefill_steps": 0, "decode_steps": 0, "decode_tokens": 0, "prefill_tokens": 0,
                      "spec_drafted": 0, "spec_accepted": 0, "spec_paused_steps": 0, "swapped_out": 0,
                      "swapped_in": 0}
        self._spec_pause = 0           # plain decode steps left before drafting again
        self._spec_recent: deque = deque()  # (drafted, accepted) of recent verify steps
        self._vocab_bytes = None  # token byte strings for constrained decoding (set_tokenizer)
        self._trie = None

    def set_tokenizer(self, tokenizer):
        """Vocabulary of the tokenizer in use, for grammar-constrained requests."""
        from ..text.constrain import vocab_bytes
        self._vocab_bytes = vocab_bytes(tokenizer, self.cfg.vocab)
        self._trie = None

    def _token_trie(self):
        if self._trie is None:
            from ..text.constrain import vocab_bytes
            vb = self._vocab_bytes if self._vocab_bytes is not None else vocab_bytes(None, self.cfg.vocab)
            self._trie = ext().TokenTrie(vb)
        return self._trie

    # ------------------------------------------------------------------ intake
    def add_request(self, prompt: list[int], params: SamplingParams | None = None, choice_index: int = 0) -> int:
        params = params or SamplingParams()
        if not prompt:
            raise ValueError("empty prompt")
        for t in prompt:
            if not 0 <= t < self.cfg.vocab:
                raise ValueError(f"token id {t} out of range [0, {self.cfg.vocab})")
        if len(prompt) + params.max_tokens > self.runner.max_seq_len:
            raise ValueError("prompt + max_tokens exceeds max_seq_len")
        if params.logprobs is not None:
            # the alternatives per token are capped like the OpenAI API's (0..20) and never
            # beyond the vocabulary; speculative steps and pipeline stages do not record them
            n = params.logprobs
            if isinstance(n, bool) or not isinstance(n, int) or not 0 <= n <= min(MAX_LOGPROBS, self.cfg.vocab):
                raise ValueError(f"logprobs: an integer count in 0..{min(MAX_LOGPROBS, self.cfg.vocab)}")
            if self.spec is not None:
                raise ValueError("logprobs are not recorded with speculative decoding")
            if self.runner.pp is not None:
                raise ValueError("logprobs are not recorded under pipeline parallelism")
        kv = self.runner.kv
        pool = kv.alloc.num_blocks - kv.alloc.reserved
        if kv.blocks_needed(len(prompt) + params.max_tokens) > pool:
            # a request must be able to finish alone (preemption makes room for it, never more)
            raise ValueError(f"prompt + max_tokens needs {kv.blocks_needed(len(prompt) + params.max_tokens)} KV "
                             f"pages; the cache has {pool}")
        if params.logit_bias and not all(0 <= int(t) < self.cfg.vocab for t in params.logit_bias):
            raise ValueError(f"logit_bias token ids must be in [0, {self.cfg.vocab})")
        if params.repetition_penalty <= 0:
            raise ValueError("repetition_penalty must be > 0")
        sid = next(self._ids)
        s = Sequence(sid, list(prompt), params, t_arrival=time.perf_counter())
        if params.constraint is not None:
            from ..text.constrain import make_constraint
            s.constraint = make_constraint(self._token_trie(), self.eos, params.constraint)
        if params.seed is not None:  # client seed: key (seed, choice index)
            s.seed, s.stream = params.seed, choice_index
        else:  # generated seed: key (seed, sequence id)
            s.seed, s.stream = self._boot_seed ^ sid, sid
        self.waiting.append(s)
        return sid

    def abort(self, seq_id: int):
        for s in list(self.prefilling):
            if s.seq_id == seq_id:
                # its pages hold only part of the prompt: returned, never published as a prefix
                self.prefilling.remove(s)
                self.runner.kv.release(s.blocks)
                s.blocks = []
                self._finish(s, "cancelled")
                return
        for item in list(self.swapped):
            if item[0].seq_id == seq_id:
                self.swapped.remove(item)
                self.kv_store.drop(item[1])
                self._finish(item[0], "cancelled")
                return
        for s in list(self.waiting):
            if s.seq_id == seq_id:
                self.waiting.remove(s)
                self._finish(s, "cancelled")
                return
        for s in self.running:
            if s.seq_id == seq_id:
                self._finish(s, "cancelled")
                self.running.remove(s)
                return

    # ------------------------------------------------------------------ saved sessions
    def save_session(self, seq_id: int) -> dict:
        """Snapshot of a running sequence: its tokens, sampling state and KV pages (packed per
        layer on the device, then copied to host memory).  `restore_session` continues it,
        in this engine or a fresh one over the same model, without a re-prefill."""
        s = next((x for x in self.running if x.seq_id == seq_id), None)
        if s is None:
            raise KeyError(f"no running sequence {seq_id}")
        kv = self.runner.kv
        layers = self._pack_kv(s)
        cfg = self.cfg
        return {"model": cfg.name, "n_layers": len(kv.k), "kv_shape": tuple(kv.k[0].shape[1:]),
                "prompt": list(s.prompt), "output": list(s.output), "params": s.params, "seed": s.seed,
                "stream": s.stream, "rng_counter": s.rng_counter, "kv": layers}

    def _pack_kv(self, s: Sequence) -> list:
        """The KV pages of s (every token but the last sampled one), packed per layer on the
        device and copied to host memory."""
        kv = self.runner.kv
        n_pages = kv.blocks_needed(s.n_tokens - 1) if s.n_tokens > 1 else 0
        pages = torch.tensor(s.blocks[:n_pages], dtype=torch.int32, device=self.runner.device)
        return [ops.kv_pack(kv.k[i], kv.v[i], pages).to("cpu") for i in range(len(kv.k))]

    def _unpack_kv(self, s: Sequence, layers: list):
        kv = self.runner.kv
        n_pages = layers[0].shape[0] if layers else 0
        kv.ensure(s.blocks, s.n_tokens)
        dev = self.runner.device
        pages = torch.tensor(s.blocks[:n_pages], dtype=torch.int32, device=dev)
        for i in range(len(kv.k)):
            ops.kv_unpack(layers[i].to(dev), kv.k[i], kv.v[i], pages)

    # ------------------------------------------------------------------ preemption (KV tiering)
    def _pages_short(self) -> int:
        """KV pages the next decode step needs beyond the free pool."""
        kv = self.runner.kv
        w = 1 + (self.spec.gamma if self.spec is not None and hasattr(self.spec, "gamma") else 0)
        need = sum(max(0, kv.blocks_needed(s.n_tokens + w - 1) - len(s.blocks)) for s in self.running)
        return need - kv.alloc.num_free

    def _swap_out(self, s: Sequence):
        """Preempt s: its KV pages go to host memory (or a spill file past the host budget) and
        back to the pool; it resumes later from exactly where it stopped (no recompute)."""
        layers = self._pack_kv(s)
        # stored first: if the store fails (a spill file that cannot be written), the sequence
        # keeps its pages and stays running
        entry = self.kv_store.put(s.seq_id, layers)
        self.runner.kv.release(s.blocks)
        s.blocks = []
        s.status = "swapped"
        self.running.remove(s)
        self.swapped.append((s, entry))
        self.stats["swapped_out"] += 1

    def _swap_in(self) -> bool:
        """Resume the oldest preempted sequence if its pages fit (before any new admission)."""
        if not self.swapped or len(self.running) >= self.runner.max_batch:
            return False
        s, entry = self.swapped[0]
        kv = self.runner.kv
        need = kv.blocks_needed(s.n_tokens + 1)
        if kv.alloc.num_free < need and self.prefix is not None:
            self.prefix.evict(need - kv.alloc.num_free)  # cached prefixes give way to a preempted sequence
        if kv.alloc.num_free < need:
            return False
        self.swapped.popleft()
        self._unpack_kv(s, self.kv_store.take(entry))
        self.kv_store.refill(e for _, e in self.swapped)  # the next to resume come back into RAM
        s.status = "running"
        self.running.append(s)
        self.stats["swapped_in"] += 1
        return True

    def restore_session(self, state: dict) -> int:
        """Re-admits a saved sequence as running: allocates pages, writes its KV back and
        resumes decoding from its last token."""
        kv = self.runner.kv
        if state["model"] != self.cfg.name or state["n_layers"] != len(kv.k) or \
                tuple(state["kv_shape"]) != tuple(kv.k[0].shape[1:]):
            raise ValueError("saved session belongs to a different model or cache layout")
        sid = next(self._ids)
        s = Sequence(sid, list(state["prompt"]), state["params"], output=list(state["output"]),
                     t_arrival=time.perf_counter())
        s.seed, s.stream, s.rng_counter = state["seed"], state["stream"], state["rng_counter"]
        if s.params.constraint is not None:  # the grammar state: replay what was emitted
            from ..text.constrain import make_constraint
            s.constraint = make_constraint(self._token_trie(), self.eos, s.params.constraint)
            for t in s.output:
                if not s.constraint.advance(int(t)):
                    raise ValueError("saved session's output does not follow its constraint")
        if kv.alloc.num_free < kv.blocks_needed(s.n_tokens + 1):
            raise RuntimeError("not enough free KV pages to restore the session")
        self._unpack_kv(s, state["kv"])
        s.status = "running"
        s.t_first_token = time.perf_counter()
        self.running.append(s)
        return sid

    def has_work(self) -> bool:
        return bool(self.waiting or self.running or self.swapped or self.prefilling)

    # ------------------------------------------------------------------ steps
    def step(self) -> list[StepOutput]:
        if self.dist is not None:
            return self._step_lockstep()
        while self._swap_in():
            pass
        if self.swapped and not self.running:  # it cannot wait for pages nobody will return
            s0 = self.swapped[0][0]
            kv = self.runner.kv
            raise MemoryError(f"preempted sequence {s0.seq_id} needs {kv.blocks_needed(s0.n_tokens + 1)} KV pages; "
                              f"{kv.alloc.num_free} are free and nothing is running")
        if self.running and self._pages_short() > 0 and self.prefix is not None:
            self.prefix.evict(self._pages_short())  # unreferenced cached prefixes go first
        if self.running and self._pages_short() > 0:
            # the KV pool cannot hold the next step: preempt the newest sequences to host memory
            while len(self.running) > 1 and self._pages_short() > 0:
                self._swap_out(self.running[-1])
            return self._log(self._decode(), len(self.running), 0)
        if self.chunk_tokens is not None:
            return self._step_chunked()
        batch = self._admit() if not self.swapped else []
        if batch:
            return self._prefill(batch)
        if self.running:
            return self._decode()
        return []

    def _log(self, outs, decode_rows: int, prefill_tokens: int):
        if self.step_log is not None:
            self.step_log.append((decode_rows, prefill_tokens))
        return outs

    def _step_chunked(self) -> list[StepOutput]:
        """Decode-first step: the running sequences' decode rows, then one prefill chunk of at
        most chunk_tokens prompt tokens (partly prefilled prompts continue first, in arrival
        order, then new prompts are admitted while pages and batch rows last)."""
        outs = []
        n_dec = len(self.running)
        if self.running:
            outs += self._decode()
        budget = self.chunk_tokens
        work = []  # (sequence, first prompt position of this chunk, tokens)
        for s in self.prefilling:
            if budget <= 0:
                break
            n = min(budget, len(s.prompt) - s.prefilled)
            work.append((s, s.prefilled, n))
            budget -= n
        if budget > 0 and not self.swapped:
            kv = self.runner.kv
            while self.waiting and budget > 0 and \
                    len(self.running) + len(self.prefilling) < self.runner.max_batch:
                s = self.waiting[0]
                need = kv.blocks_needed(len(s.prompt) + 1)
                if kv.alloc.num_free < need and self.prefix is not None:
                    self.prefix.evict(need - kv.alloc.num_free)
                if kv.alloc.num_free < need:
                    break
                self.waiting.popleft()
                if self.prefix is not None:
                    s.blocks, s.cached_tokens = self.prefix.match(s.prompt)
                    # the last prompt token is always computed (its logits give the first token)
                    s.cached_tokens = min(s.cached_tokens, len(s.prompt) - 1)
                kv.ensure(s.blocks, len(s.prompt))
                s.prefilled = s.cached_tokens
                self.prefilling.append(s)
                n = min(budget, len(s.prompt) - s.prefilled)
                work.append((s, s.prefilled, n))
                budget -= n
        n_pre = sum(n for _, _, n in work)
        if work:
            outs += self._prefill_chunk(work)
        return self._log(outs, n_dec, n_pre)

    def _prefill_chunk(self, work) -> list[StepOutput]:
        kv = self.runner.kv
        toks, pos, slots, cu, prefix = [], [], [], [0], []
        for s, st, n in work:
            toks += s.prompt[st:st + n]
            pos += list(range(st, st + n))
            slots += [kv.slot(s.blocks, p) for p in range(st, st + n)]
            cu.append(cu[-1] + n)
            prefix.append((list(s.blocks), st))
        logits = self.runner.prefill(torch.tensor(toks), torch.tensor(pos), torch.tensor(slots), cu,
                                     prefix if any(p[1] for p in prefix) else None,
                                     block_lists=[list(s.blocks) for s, _, _ in work])
        self.stats["prefill_steps"] += 1
        self.stats["prefill_tokens"] += cu[-1]
        done = [i for i, (s, st, n) in enumerate(work) if st + n == len(s.prompt)]
        for s, st, n in work:
            s.prefilled = st + n
        if not done:
            return []
        seqs = [work[i][0] for i in done]
        rows = logits[done]
        nxt = self._sample_rows(rows, seqs)
        self._record_logprobs(rows, seqs, nxt)
        now = time.perf_counter()
        outs = []
        for s, t in zip(seqs, nxt):
            self.prefilling.remove(s)
            s.t_first_token = now
            s.status = "running"
            self.running.append(s)
            outs.append(self._append(s, t))
        self._reap()
        return outs

    def _step_lockstep(self) -> list[StepOutput]:
        import torch.distributed as dist
        t0 = time.perf_counter()
        want = torch.tensor([1 if self._can_admit() else 0, 1 if self.running else 0], dtype=torch.int64)
        dist.all_reduce(want, op=dist.ReduceOp.MAX, group=self.dist.cpu_group)
        self.stats["lockstep_s"] = self.stats.get("lockstep_s", 0.0) + time.perf_counter() - t0
        if want[0]:
            return self._prefill(self._admit())
        if want[1]:
            return self._decode()
        return []

    def _can_admit(self) -> bool:
        if not self.waiting or len(self.running) >= self.runner.max_batch:
            return False
        s = self.waiting[0]
        return self.runner.kv.alloc.num_free >= self.runner.kv.blocks_needed(len(s.prompt) + 1)

    def global_has_work(self) -> bool:
        if self.dist is None:
            return self.has_work()
        import torch.distributed as dist
        t = torch.tensor([1 if self.has_work() else 0], dtype=torch.int64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=self.dist.cpu_group)
        return bool(t[0])

    def _admit(self) -> list[Sequence]:
        kv = self.runner.kv
        batch, tokens = [], 0
        while self.waiting and len(self.running) + len(batch) < self.runner.max_batch:
            s = self.waiting[0]
            need = kv.blocks_needed(len(s.prompt) + 1)
            if kv.alloc.num_free < need and self.prefix is not None:
                self.prefix.evict(need - kv.alloc.num_free)
            if kv.alloc.num_free < need or (batch and tokens + len(s.prompt) > self.max_prefill_tokens):
                break
            self.waiting.popleft()
            if self.prefix is not None:
                s.blocks, s.cached_tokens = self.prefix.match(s.prompt)
            kv.ensure(s.blocks, len(s.prompt))
            batch.append(s)
            tokens += len(s.prompt) - s.cached_tokens
        return batch

    def _prefill(self, batch: list[Sequence]) -> list[StepOutput]:
        kv = self.runner.kv
        if not batch:  # lockstep participation with no local prompts
            self.runner.prefill(torch.zeros(0, dtype=torch.int32), torch.zeros(0, dtype=torch.int32),
                                torch.zeros(0, dtype=torch.int64), [0])
            return []
        toks, pos, slots, cu, prefix = [], [], [], [0], []
        for s in batch:
            st = s.cached_tokens
            toks += s.prompt[st:]
            pos += list(range(st, len(s.prompt)))
            slots += [kv.slot(s.blocks, p) for p in range(st, len(s.prompt))]
            cu.append(cu[-1] + len(s.prompt) - st)
            prefix.append((list(s.blocks), st))
        logits = self.runner.prefill(torch.tensor(toks), torch.tensor(pos), torch.tensor(slots), cu,
                                     prefix if any(p[1] for p in prefix) else None,
                                     block_lists=[list(s.blocks) for s in batch])
        pp = self.runner.pp
        if pp is not None:
            toks_t = torch.zeros(len(batch), dtype=torch.int32, device=self.runner.device)
            if pp.last:
                toks_t.copy_(torch.tensor(self._sample_rows(logits, batch), dtype=torch.int32))
            else:
                for s in batch:  # keep the draw counters in step with the sampling stage
                    if s.params.temperature > 0:
                        s.rng_counter += 1
            nxt = pp.broadcast_tokens(toks_t).cpu().tolist()
        else:
            nxt = self._sample_rows(logits, batch)
            self._record_logprobs(logits, batch, nxt)
        self.stats["prefill_steps"] += 1
        self.stats["prefill_tokens"] += cu[-1]
        now = time.perf_counter()
        outs = []
        for s, t in zip(batch, nxt):
            s.t_first_token = now
            s.status = "running"
            self.running.append(s)
            outs.append(self._append(s, t))
        if self.spec is not None and hasattr(self.spec.drafter, "after_prefill"):
            self.spec.drafter.after_prefill(batch, self.runner._prefill_x, cu)
        self._reap()
        return outs

    @staticmethod
    def _record_logprobs(logits: torch.Tensor, seqs: list[Sequence], toks: list[int]):
        """Log-softmax (f32) of the rows that asked for logprobs: the emitted token's value and
        the top alternatives.  Rows that did not ask cost nothing."""
        rows = [i for i, s in enumerate(seqs) if s.params.logprobs is not None]
        if not rows:
            return
        lp = torch.log_softmax(logits[rows].float(), -1)
        chosen = lp.gather(1, torch.tensor([toks[i] for i in rows], device=lp.device)[:, None])[:, 0].cpu().tolist()
        k = min(max(seqs[i].params.logprobs for i in rows), lp.shape[-1])
        tv, ti = lp.topk(k, -1) if k else (None, None)
        tv, ti = (tv.cpu().tolist(), ti.cpu().tolist()) if k else ([], [])
        for j, i in enumerate(rows):
            n = seqs[i].params.logprobs
            seqs[i].logprobs.append({"token": int(toks[i]), "logprob": chosen[j],
                                     "top": [(int(t), v) for t, v in zip(ti[j][:n], tv[j][:n])] if n else []})

    @staticmethod
    def _redraw(s: Sequence) -> bool:
        return s.constraint is not None or s.params.processed

    @staticmethod
    def _process_logits(row: torch.Tensor, s: Sequence):
        """In place on one row: penalties over the tokens seen so far, then logit bias
        (OpenAI / HF semantics; reference LogitsProcess, crates/kernels/src/op/kind.rs)."""
        p = s.params
        dev = row.device
        if p.repetition_penalty != 1.0:
            seen = torch.tensor(sorted(set(s.prompt) | set(s.output)), dtype=torch.long, device=dev)
            v = row[seen]
            row[seen] = torch.where(v > 0, v / p.repetition_penalty, v * p.repetition_penalty)
        if (p.frequency_penalty or p.presence_penalty) and s.output:
            ids, cnt = torch.unique(torch.tensor(s.output, dtype=torch.long), return_counts=True)
            row[ids.to(dev)] -= (p.frequency_penalty * cnt.float() + p.presence_penalty).to(dev)
        if p.logit_bias:
            ids = torch.tensor([int(k) for k in p.logit_bias], dtype=torch.long, device=dev)
            row[ids] += torch.tensor([float(v) for v in p.logit_bias.values()], device=dev)

    def _sample_rows(self, logits: torch.Tensor, seqs: list[Sequence]) -> list[int]:
        n = len(seqs)
        dev = logits.device
        if any(self._redraw(s) for s in seqs):
            # penalties / bias, then the grammar: forbidden tokens of constrained rows at -inf
            from ..text.constrain import allowed
            logits = logits.clone()
            for i, s in enumerate(seqs):
                if s.params.processed:
                    self._process_logits(logits[i], s)
                if s.constraint is not None:
                    logits[i].masked_fill_(~allowed(s.constraint.mask(), logits.shape[1]).to(dev), float("-inf"))
        temp = torch.tensor([s.params.temperature for s in seqs], dtype=torch.float32, device=dev)
        topk = torch.tensor([s.params.top_k for s in seqs], dtype=torch.int32, device=dev)
        topp = torch.tensor([s.params.top_p for s in seqs], dtype=torch.float32, device=dev)
        seed = torch.tensor([s.seed for s in seqs], dtype=torch.int64, device=dev)
        stream = torch.tensor([s.stream for s in seqs], dtype=torch.int64, device=dev)
        ctr = torch.tensor([s.rng_counter for s in seqs], dtype=torch.int64, device=dev)
        out = torch.empty(n, dtype=torch.int32, device=dev)
        ops.sample(logits.contiguous(), temp, topk, topp, seed, stream, ctr, out)
        ctr_h = ctr.cpu().tolist()
        for s, c in zip(seqs, ctr_h):
            s.rng_counter = int(c)
        return out.cpu().tolist()

    def _decode(self) -> list[StepOutput]:
        # Under lockstep ranks every rank runs the same verify window shape (equal live
        # sequence counts), so the expert-parallel exchanges inside it line up.
        if self.spec is None:
            outs = self._decode_plain()
        elif self._spec_pause > 0:
            self._spec_pause -= 1
            self.stats["spec_paused_steps"] += 1
            outs = self._decode_plain()
        else:
            d0, a0 = self.stats["spec_drafted"], self.stats["spec_accepted"]
            outs = self._decode_spec()
            self._spec_adapt(self.stats["spec_drafted"] - d0, self.stats["spec_accepted"] - a0)
        r = self.runner
        n = self.stats["decode_steps"]
        if r.expert_cache is not None and self.rebalance_every and n % self.rebalance_every == 0:
            r.adapt_experts()  # lockstep ranks reach the same step count together
        return outs

    def _decode_spec(self) -> list[StepOutput]:
        """One verify window per sequence: rows [last, d1..dg] at positions p..p+g."""
        from .spec import verify
        r, kv, g = self.runner, self.runner.kv, self.spec.gamma
        seqs = self.running[: max(1, r.max_batch // (g + 1))]
        rows = len(seqs) * (g + 1)
        d = r.desc.h
        drafts = []
        mtp = hasattr(self.spec.drafter, "after_verify")
        stochastic = getattr(self.spec.drafter, "stochastic", False)
        probs = []  # stochastic drafts: the distribution each was sampled from
        batch = getattr(self.spec.drafter, "propose_batch", None)
        if batch is not None and not mtp and not stochastic:
            drafts = batch([s.prompt + s.output for s in seqs], g)
        else:
            for s in seqs:
                if mtp:
                    dr = (s.mtp_draft or [s.output[-1]])[:g]
                elif stochastic:
                    dr, q = self.spec.drafter.propose(s.prompt + s.output, g, key=s.seq_id, seed=s.seed ^ s.stream)
                    probs.append(q)
                elif getattr(self.spec.drafter, "stateful", False):
                    dr = self.spec.drafter.propose(s.prompt + s.output, g, key=s.seq_id)
                else:
                    dr = self.spec.drafter.propose(s.prompt + s.output, g)
                drafts.append(dr)
        # every verify row of every window in one native descriptor fill (greedy rows: the
        # acceptance draws on the host-side verify, not in the graph's sampler)
        tok_rows, pos_rows, slot_rows, bl_rows = [], [], [], []
        for s, dr in zip(seqs, drafts):
            p = s.n_tokens - 1
            kv.ensure(s.blocks, p + g + 1)
            for j, tok in enumerate([s.output[-1]] + list(dr)):
                tok_rows.append(int(tok))
                pos_rows.append(p + j)
                slot_rows.append(kv.slot(s.blocks, p + j))
                bl_rows.append(s.blocks)
        from .runner import bucket_for
        zeros_i, zeros_l = [0] * rows, [0] * rows
        ext().step_desc_fill(r.desc.host, r.desc.rows, r.desc.max_blocks, tok_rows, pos_rows, zeros_i, slot_rows,
                             zeros_l, zeros_l, zeros_l, [0.0] * rows, [1.0] * rows, bl_rows,
                             bucket_for(rows, cap=r.max_batch) if r.use_graphs else rows)
        r.decode(rows)
        logits = r.buf["logits"][:rows]
        temp = torch.tensor([s.params.temperature for s in seqs], dtype=torch.float32)
        topk = torch.tensor([s.params.top_k for s in seqs], dtype=torch.int32)
        topp = torch.tensor([s.params.top_p for s in seqs], dtype=torch.float32)
        seed = torch.tensor([s.seed for s in seqs], dtype=torch.int64)
        stream = torch.tensor([s.stream for s in seqs], dtype=torch.int64)
        ctr = torch.tensor([s.rng_counter for s in seqs], dtype=torch.int64)
        toks, nacc = verify(logits, torch.tensor(drafts, dtype=torch.int32), temp, topk, topp, seed, stream, ctr,
                            torch.stack(probs) if stochastic else None)
        r.after_step()
        redo = [i for i, s in enumerate(seqs) if self._redraw(s)]
        if redo:
            # penalised / constrained rows take one token per step, drawn from their processed
            # logits at the window's first row with their own counter (exactly a plain step), so
            # what the others in the batch do never changes their draws; their drafts are dropped
            t1 = self._sample_rows(logits[[i * (g + 1) for i in redo]], [seqs[i] for i in redo])
            for i, t in zip(redo, t1):
                toks[i, 0], nacc[i], ctr[i] = t, 0, seqs[i].rng_counter
        self.stats["decode_steps"] += 1
        outs = []
        mtp_items = []
        for i, s in enumerate(seqs):
            s.rng_counter = int(ctr[i])
            n = int(nacc[i])
            if mtp:
                row = i * (g + 1) + n
                mtp_items.append((s, r.buf["x"][row].clone(), int(d["pos"][row])))
            if i not in redo:
                self.stats["spec_drafted"] += g
                self.stats["spec_accepted"] += n
            new = toks[i, : n + 1].tolist()
            emitted = []
            for t in new:
                o = self._append(s, t)
                emitted.append(t)
                if o.finished:
                    break
            self.stats["decode_tokens"] += len(emitted)
            outs.append(StepOutput(s.seq_id, emitted, s.status == "finished", s.finish_reason))
        if mtp:
            self.spec.drafter.after_verify(mtp_items)
        self._reap()
        return outs

    def _spec_adapt(self, drafted: int, accepted: int):
        """Pauses drafting for a while when recent acceptance is too low to pay for the verify
        windows (point-mass drafters on one rank only)."""
        sp = self.spec
        if sp.min_accept <= 0 or self.dist is not None or hasattr(sp.drafter, "after_verify") or \
                getattr(sp.drafter, "stochastic", False):
            return
        self._spec_recent.append((drafted, accepted))
        tot = sum(d for d, _ in self._spec_recent)
        while self._spec_recent and tot - self._spec_recent[0][0] >= sp.window:
            tot -= self._spec_recent.popleft()[0]
        if tot >= sp.window and sum(a for _, a in self._spec_recent) < sp.min_accept * tot:
            self._spec_pause = sp.pause_steps
            self._spec_recent.clear()

    @property
    def acceptance_rate(self) -> float:
        return self.stats["spec_accepted"] / max(1, self.stats["spec_drafted"])

    def _decode_plain(self) -> list[StepOutput]:
        r = self.runner
        kv = r.kv
        seqs = self.running
        B = len(seqs)
        pos = []
        for s in seqs:
            p = s.n_tokens - 1
            kv.ensure(s.blocks, p + 1)
            pos.append(p)
        from .runner import bucket_for
        # one native call writes every live row and the bucket's padding rows
        ext().step_desc_fill(r.desc.host, r.desc.rows, r.desc.max_blocks, [s.output[-1] for s in seqs], pos,
                             [s.params.top_k for s in seqs], [kv.slot(s.blocks, p) for s, p in zip(seqs, pos)],
                             [s.seed for s in seqs], [s.stream for s in seqs], [s.rng_counter for s in seqs],
                             [float(s.params.temperature) for s in seqs], [float(s.params.top_p) for s in seqs],
                             [s.blocks for s in seqs], bucket_for(B, cap=r.max_batch) if r.use_graphs else B)
        nxt = r.decode(B).cpu().tolist()
        r.after_step()
        cons = [i for i, s in enumerate(seqs) if self._redraw(s)]
        if cons:  # constrained / processed rows draw again from their processed logits, same counter
            redo = self._sample_rows(r.buf["logits"][:B][cons], [seqs[i] for i in cons])
            for i, t in zip(cons, redo):
                nxt[i] = t
        self._record_logprobs(r.buf["logits"][:B], seqs, nxt)
        # greedy rows take no draw; sampled rows take exactly one (re-drawn rows took theirs)
        for s in seqs:
            if s.params.temperature > 0 and not self._redraw(s):
                s.rng_counter += 1
        self.stats["decode_steps"] += 1
        self.stats["decode_tokens"] += B
        outs = [self._append(s, t) for s, t in zip(seqs, nxt)]
        self._reap()
        return outs

    def _append(self, s: Sequence, tok: int) -> StepOutput:
        s.output.append(int(tok))
        reason = None
        if s.constraint is not None:  # the masked sampler only picks tokens the grammar allows
            if self.eos is not None and tok == self.eos:
                reason = "stop"
            else:
                s.constraint.advance(int(tok))
                if s.constraint.finished():
                    reason = "stop"
        if reason is None and len(s.output) >= s.params.max_tokens:
            reason = "length"
        elif reason is None and (tok in s.params.stop_token_ids or
                                 (not s.params.ignore_eos and self.eos is not None and tok == self.eos)):
            reason = "stop"
        if reason:
            s.finish_reason = reason
            s.status = "finished"
        lp = s.logprobs[-1:] if s.params.logprobs is not None and len(s.logprobs) == len(s.output) else None
        return StepOutput(s.seq_id, [int(tok)], reason is not None, reason, lp)

    def _finish(self, s: Sequence, reason: str):
        s.status = "finished"
        s.finish_reason = s.finish_reason or reason
        s.t_finished = time.perf_counter()
        if self.prefix is not None and s.blocks:
            # KV holds every token but the last sampled one
            self.prefix.insert((s.prompt + s.output)[: s.n_tokens - 1], s.blocks)
        self.runner.kv.release(s.blocks)
        if self.spec is not None and hasattr(self.spec.drafter, "release"):
            self.spec.drafter.release(s.seq_id)
        self.finished[s.seq_id] = s

    def _reap(self):
        keep = []
        for s in self.running:
            if s.status == "finished":
                self._finish(s, s.finish_reason or "length")
            else:
                keep.append(s)
        self.running = keep

    # ------------------------------------------------------------------ convenience
    def generate(self, prompts: list[list[int]], params: SamplingParams | list[SamplingParams]) -> list[list[int]]:
        plist = params if isinstance(params, list) else [params] * len(prompts)
        ids = [self.add_request(p, sp) for p, sp in zip(prompts, plist)]
        while self.global_has_work():
            self.step()
        return [self.finished[i].output for i in ids]
