"""CPU: the KV arena allocator and the continuous-batching scheduler's policy
(admission, chunked prefill budget, slot reuse, stopping rules), driven by a
fake engine and a fake slot decoder whose next token is a known function of
the input.  No kernel is launched here."""
from __future__ import annotations

import importlib

import pytest
import torch

from conftest import ROOT  # noqa: F401  (puts the repository on sys.path)

pool_mod = importlib.import_module("roofline-inference_b200.pool")
sched_mod = importlib.import_module("roofline-inference_b200.scheduler")
KVPool, PoolFull = pool_mod.KVPool, pool_mod.PoolFull
VOCAB = 1000


# ------------------------------------------------------------------ allocator
def test_pool_best_fit_and_coalescing():
    p = KVPool(2, 1, rows=10 * 256, head_dim=8)
    a = p.allocate(300)                 # 2 pages
    b = p.allocate(256)                 # 1 page
    c = p.allocate(700)                 # 3 pages
    assert (a.capacity, b.capacity, c.capacity) == (512, 256, 768)
    assert p.free_pages == 4
    # the views are disjoint ranges of the arena, laid out like a stand-alone Cache
    assert tuple(a.storage.shape) == (2, 2, 1, 512, 8)
    a.storage.fill_(1)
    c.storage.fill_(3)
    assert float(b.storage.abs().sum()) == 0.0
    p.free(b)                           # hole of 1 page between a and c
    d = p.allocate(200)                 # best fit: the 1-page hole, not the 4-page tail
    assert d.storage.data_ptr() == a.storage.data_ptr() + a.storage.numel() * 2
    p.free(a)
    p.free(d)                           # a + d merge into 3 pages at the start
    e = p.allocate(3 * 256)
    assert e.storage.data_ptr() == p.arena.data_ptr()
    p.free(e)
    p.free(c)
    assert p._free == [(0, 10)] and p.free_pages == 10
    with pytest.raises(ValueError):
        p.free(c)                       # double free


def test_pool_full_and_fragmentation():
    p = KVPool(1, 1, rows=4 * 256, head_dim=8)
    xs = [p.allocate(256) for _ in range(4)]
    with pytest.raises(PoolFull):
        p.allocate(1)
    p.free(xs[0])
    p.free(xs[2])
    assert p.free_pages == 2 and p.largest_free_rows == 256
    with pytest.raises(PoolFull):
        p.allocate(512)                 # two free pages, not adjacent
    p.free(xs[1])
    assert p.allocate(768).capacity == 768


def test_cache_over_rejects_bad_storage():
    cache_mod = importlib.import_module("roofline-inference_b200.cache")
    with pytest.raises(ValueError):
        cache_mod.Cache.over(torch.zeros(2, 2, 1, 100, 8))


# ------------------------------------------------------------------ scheduler
class FakeCfg:
    vocab_size = VOCAB


class FakeEngine:
    """prefill advances the cache offset; the last chunk's logits peak at
    (sum of the prompt) % VOCAB."""

    def __init__(self):
        self.cfg, self.device = FakeCfg(), torch.device("cpu")
        self.calls = []
        self.seen: dict[int, list[int]] = {}

    def prefill(self, toks, cache, last):
        n = int(toks.numel())
        if cache.offset + n > cache.capacity:
            raise ValueError("KV capacity exceeded")
        self.calls.append(n)
        if cache.offset == 0:               # a new request (a freed cache's id can come back)
            self.seen[id(cache)] = []
        self.seen[id(cache)].extend(toks.tolist())
        cache.offset += n
        if not last:
            return None
        lg = torch.zeros(VOCAB)
        lg[sum(self.seen[id(cache)]) % VOCAB] = 1.0
        return lg


class FakeDecoder:
    """next token = (input + 1) % VOCAB for every active slot."""

    def __init__(self, slots):
        self.caches = [None] * slots
        self.tok = [0] * slots
        self.graph = None

    def free_slots(self):
        return [i for i, c in enumerate(self.caches) if c is None]

    def set_slot(self, i, cache, token):
        assert self.caches[i] is None
        self.caches[i], self.tok[i] = cache, int(token)

    def clear_slot(self, i):
        c, self.caches[i] = self.caches[i], None
        return c

    def run_step(self):
        for i, c in enumerate(self.caches):
            if c is not None:
                assert c.offset + 1 <= c.capacity
                c.offset += 1
                self.tok[i] = (self.tok[i] + 1) % VOCAB
        return torch.tensor(self.tok, dtype=torch.int32)


def make(slots=2, rows=16 * 256, chunk=64, max_len=4096):
    eng = FakeEngine()
    pool = KVPool(1, 1, rows=rows, head_dim=8)
    s = sched_mod.Scheduler(eng, pool_rows=rows, slots=slots, max_len=max_len, chunk=chunk, use_graph=False,
                            pool=pool, decoder=FakeDecoder(slots),
                            argmax_fn=lambda x: torch.argmax(x).reshape(1))
    return s, eng


def expected(prompt, max_tokens, eos=()):
    t, out = sum(prompt) % VOCAB, []
    while len(out) < max_tokens:
        out.append(t)
        if t in eos:
            break
        t = (t + 1) % VOCAB
    return out


def test_scheduler_matches_single_stream_order():
    s, _ = make(slots=2)
    prompts = [[5, 6, 7], [100] * 40, [1], [9, 9], [3] * 130]
    mts = [4, 7, 1, 5, 3]
    ids = [s.submit(p, m) for p, m in zip(prompts, mts)]
    out = s.run()
    for i, p, m in zip(ids, prompts, mts):
        assert out[i] == expected(p, m), i
        assert s.finished[i].reason == "length"
    assert s.pool.free_pages == s.pool.pages          # every cache returned
    assert not s.running and all(c is None for c in s.dec.caches)


def test_scheduler_eos_and_zero_tokens():
    s, _ = make(slots=4)
    a = s.submit([10, 20], max_tokens=50, eos_ids=[33])        # first token 30: 30, 31, 32, 33 stop
    b = s.submit([1, 2], max_tokens=0)
    c = s.submit([2], max_tokens=1)                           # the prefill token only, no decode slot
    out = s.run()
    assert out[a] == [30, 31, 32, 33] and s.finished[a].reason == "eos"
    assert out[b] == [] and out[c] == [2]


def test_scheduler_chunked_prefill_budget():
    s, eng = make(slots=2, chunk=64)
    s.submit([1] * 150, max_tokens=2)
    s.submit([2] * 10, max_tokens=2)
    s.step()
    assert eng.calls == [64]                  # one chunk per step over all requests
    s.step()
    assert eng.calls == [64, 64]
    s.step()                                  # 22 tokens finish the first prompt, 10 the second
    assert eng.calls == [64, 64, 22, 10]
    out = s.run()
    assert out[0] == expected([1] * 150, 2) and out[1] == expected([2] * 10, 2)


def test_scheduler_waits_for_pool_space():
    # room for one 512-row cache at a time: requests run one after another
    s, _ = make(slots=4, rows=2 * 256)
    ids = [s.submit([7] * 300, max_tokens=3) for _ in range(3)]
    s.step()
    assert len(s.waiting) == 2
    out = s.run()
    assert all(out[i] == expected([7] * 300, 3) for i in ids)
    # a request larger than the whole pool can never run
    s2, _ = make(slots=1, rows=256)
    s2.submit([1] * 300, max_tokens=1)
    with pytest.raises(PoolFull):
        s2.run()


def test_scheduler_argument_checks():
    s, _ = make(max_len=512)
    with pytest.raises(ValueError):
        s.submit([], 3)
    with pytest.raises(ValueError):
        s.submit([VOCAB], 3)
    with pytest.raises(ValueError):
        s.submit([1], -1)
    with pytest.raises(ValueError):
        s.submit([1] * 500, 20)               # capacity above max_len
    # a rejected request takes no id: accepted ones stay consecutive
    assert [s.submit([1, 2], 3), s.submit([3], 2)] == [0, 1]


# ------------------------------------------------------------------ randomized
def test_pool_random_alloc_free_invariants():
    """Random allocate / free sequences: live blocks never overlap, the free
    list stays sorted and fully merged, and free + used pages always add up
    to the arena."""
    import random
    rng = random.Random(7)
    p = KVPool(1, 1, rows=64 * 256, head_dim=8)
    live = []
    for _ in range(2000):
        if live and (rng.random() < 0.45 or p.free_pages == 0):
            c = live.pop(rng.randrange(len(live)))
            p.free(c)
        else:
            want = rng.randint(1, 12 * 256)
            try:
                live.append(p.allocate(want))
            except PoolFull:
                assert p.largest_free_rows < want
                continue
        spans = sorted((c.storage.data_ptr(), c.storage.data_ptr() + c.storage.numel() * 2) for c in live)
        for (a0, a1), (b0, _) in zip(spans, spans[1:]):
            assert a1 <= b0
        starts = [s for s, _ in p._free]
        assert starts == sorted(starts)
        for (s0, n0), (s1, _) in zip(p._free, p._free[1:]):
            assert s0 + n0 < s1                      # adjacent free blocks are merged
        used = sum(c.capacity // 256 for c in live)
        assert used + p.free_pages == p.pages
    for c in live:
        p.free(c)
    assert p._free == [(0, 64)]


def test_scheduler_random_workload_matches_single_stream():
    """Random prompts, output lengths, end-of-sequence ids, slot counts, pool
    sizes and chunk sizes: every request gets exactly the single-stream
    greedy tokens, every cache and slot is returned, and the chunk budget per
    step is never exceeded."""
    import random
    rng = random.Random(11)
    for trial in range(25):
        slots = rng.randint(1, 5)
        chunk = rng.choice([16, 64, 100, 4096])
        rows = rng.randint(4, 24) * 256
        s, eng = make(slots=slots, rows=rows, chunk=chunk, max_len=rows)
        reqs = []
        for _ in range(rng.randint(1, 12)):
            n = rng.randint(1, 300)
            m = rng.randint(0, 40)
            if n + m + 1 > rows:
                continue
            prompt = [rng.randrange(VOCAB) for _ in range(n)]
            eos = [rng.randrange(VOCAB)] if rng.random() < 0.5 else []
            reqs.append((s.submit(prompt, m, eos), prompt, m, eos))
        before = len(eng.calls)
        steps_before = s.steps
        out = s.run()
        for rid, prompt, m, eos in reqs:
            assert out[rid] == expected(prompt, m, eos), (trial, rid)
        assert s.pool.free_pages == s.pool.pages
        assert all(c is None for c in s.dec.caches)
        # prompt tokens per step never exceed the chunk
        per_step = eng.calls[before:]
        assert all(c <= chunk for c in per_step)
        assert sum(per_step) == sum(len(p) for _, p, m, _ in reqs if m > 0)
        assert s.steps >= steps_before
