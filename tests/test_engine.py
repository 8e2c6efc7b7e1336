"""Micro-batch scheduler (EmbeddingEngine) on a fake runtime, no GPU.

The first two tests restate tests/embedding-engine.test.ts of the reference
(coalescing 16 requests in order; EOS padding after each request's final
token); the rest cover the varlen packing and the flush/error behaviour of
src/webgpu/embedding-engine.ts:56-87.
"""
import asyncio
import importlib

import numpy as np
import pytest

engine_mod = importlib.import_module("qwen3-embedding-webgpu-prepacked_b200.engine")
EmbeddingEngine = engine_mod.EmbeddingEngine


class Ids:
    def __init__(self, rows):
        self.rows = rows

    def tolist(self):
        return self.rows


class Tok:
    def __init__(self, rows):
        self.input_ids = Ids(rows)


def number_tokenizer(text):
    return Tok([[int(t) for t in text.split(",")]])


class FakeRuntime:
    def __init__(self, fail=False):
        self.calls = []
        self.plans_made = []
        self.fail = fail

    def create_plan(self, batch, sequence):
        self.plans_made.append(("padded", batch, sequence))
        rt = self

        class Plan:
            async def run(self, ids, lengths):
                rt.calls.append({"batch": batch, "sequence": sequence, "ids": list(ids),
                                 "lengths": list(lengths)})
                if rt.fail:
                    raise RuntimeError("device lost")
                return [np.array([ids[i * sequence]], np.float32) for i in range(batch)]
        return Plan()

    def create_varlen_plan(self, batch, capacity):
        self.plans_made.append(("varlen", batch, capacity))
        rt = self

        class Plan:
            def run_varlen(self, ids, cu):
                rt.calls.append({"batch": batch, "capacity": capacity, "ids": list(ids),
                                 "cu": list(cu)})
                # embedding = (first token, length) of each request
                return [np.array([ids[cu[i]], cu[i + 1] - cu[i]], np.float32)
                        for i in range(batch)]
        return Plan()


def run(coro):
    return asyncio.run(coro)


def test_coalesces_16_requests_and_preserves_order():
    rt = FakeRuntime()

    async def main():
        eng = EmbeddingEngine(rt, lambda t: Tok([[int(t)]]), 16)
        return await asyncio.gather(*[eng.embed(str(i + 1)) for i in range(16)])

    results = run(main())
    assert len(rt.calls) == 1
    c = rt.calls[0]
    assert c["batch"] == 16 and c["sequence"] == 2 and c["lengths"] == [2] * 16
    assert [float(r[0]) for r in results] == list(range(1, 17))


def test_pads_mixed_lengths_after_final_token():
    rt = FakeRuntime()

    async def main():
        eng = EmbeddingEngine(rt, number_tokenizer, 16, 0, 99)
        await asyncio.gather(eng.embed("1"), eng.embed("2,3"))

    run(main())
    assert rt.calls[0]["ids"] == [1, 99, 99, 2, 3, 99]


def test_eos_not_duplicated():
    rt = FakeRuntime()

    async def main():
        eng = EmbeddingEngine(rt, number_tokenizer, 16, 0, 99)
        await eng.embed("5,99")

    run(main())
    assert rt.calls[0]["ids"] == [5, 99] and rt.calls[0]["lengths"] == [2]


def test_max_batch_size_bounds():
    for bad in (0, 17):
        with pytest.raises(ValueError):
            EmbeddingEngine(FakeRuntime(), number_tokenizer, bad)
    with pytest.raises(ValueError):
        EmbeddingEngine(FakeRuntime(), number_tokenizer, 4, packing="nested")


def test_more_than_max_batch_splits_in_arrival_order_and_caches_plans():
    rt = FakeRuntime()

    async def main():
        eng = EmbeddingEngine(rt, number_tokenizer, 4, 0, 99)
        res = await asyncio.gather(*[eng.embed(str(i)) for i in range(1, 11)])
        # a second wave with the same shapes reuses the cached plans
        res2 = await asyncio.gather(*[eng.embed(str(i)) for i in range(1, 5)])
        return res, res2, eng

    res, res2, eng = run(main())
    assert [c["batch"] for c in rt.calls] == [4, 4, 2, 4]
    assert [float(r[0]) for r in res] == list(range(1, 11))
    assert [float(r[0]) for r in res2] == [1, 2, 3, 4]
    assert rt.plans_made == [("padded", 4, 2), ("padded", 2, 2)]
    assert set(eng.plans) == {(4, 2), (2, 2)}


def test_error_rejects_whole_micro_batch_and_engine_recovers():
    rt = FakeRuntime(fail=True)

    async def main():
        eng = EmbeddingEngine(rt, number_tokenizer, 16, 0, 99)
        outs = await asyncio.gather(eng.embed("1"), eng.embed("2"), return_exceptions=True)
        rt.fail = False
        ok = await eng.embed("3")
        return outs, ok

    outs, ok = run(main())
    assert all(isinstance(o, RuntimeError) and "device lost" in str(o) for o in outs)
    assert float(ok[0]) == 3


def test_varlen_packs_without_padding():
    rt = FakeRuntime()

    async def main():
        eng = EmbeddingEngine(rt, number_tokenizer, 16, 0, 99, packing="varlen")
        return await asyncio.gather(eng.embed("1"), eng.embed("2,3"), eng.embed("4,5,6,7"))

    res = run(main())
    c = rt.calls[0]
    assert c["ids"] == [1, 99, 2, 3, 99, 4, 5, 6, 7, 99]
    assert c["cu"] == [0, 2, 5, 10]
    assert c["capacity"] == 256
    assert [tuple(map(float, r)) for r in res] == [(1, 2), (2, 3), (4, 5)]


def test_varlen_capacity_buckets():
    cap = engine_mod.capacity_for
    assert cap(1) == 256 and cap(256) == 256 and cap(257) == 512 and cap(80000) == 131072


def test_batch_window_coalesces_staggered_requests():
    rt = FakeRuntime()

    async def main():
        eng = EmbeddingEngine(rt, number_tokenizer, 16, 50, 99)
        f1 = eng.embed("1")
        await asyncio.sleep(0.01)
        f2 = eng.embed("2")
        return await asyncio.gather(f1, f2)

    run(main())
    assert len(rt.calls) == 1 and rt.calls[0]["batch"] == 2


def test_requests_arriving_during_flush_are_served():
    rt = FakeRuntime()

    async def main():
        eng = EmbeddingEngine(rt, number_tokenizer, 2, 0, 99)
        first = [eng.embed("1"), eng.embed("2")]
        await asyncio.sleep(0)  # let the flush start
        late = eng.embed("3")
        return await asyncio.gather(*first, late)

    res = run(main())
    assert [float(r[0]) for r in res] == [1, 2, 3]


def test_assemblers_match_reference_layout():
    eng = EmbeddingEngine(FakeRuntime(), number_tokenizer, 16, 0, 7)
    ids, lengths, seq = eng.assemble_padded([[1, 7], [2, 3, 4, 7]])
    assert seq == 4 and list(ids) == [1, 7, 7, 7, 2, 3, 4, 7] and list(lengths) == [2, 4]
    ids, cu = EmbeddingEngine.assemble_varlen([[1, 7], [2, 3, 4, 7]])
    assert list(ids) == [1, 7, 2, 3, 4, 7] and list(cu) == [0, 2, 6]
