"""Host-side logic without a GPU: allocator, tables, rollback, scheduler, configs.

Cases follow reference tests/test_cache.py and tests/test_scheduler.py.
"""

from __future__ import annotations

import numpy as np
import pytest

from microserve_b200.cache import BlockAllocator, OutOfCacheMemory, PagedKVCache
from microserve_b200.config import (CacheConfig, EngineConfig, ModelConfig, SamplingConfig,
                                    SchedulerConfig, SpeculativeConfig, load_config)
from microserve_b200.scheduler import Request, Scheduler

from .conftest import ROOT


def host_cache(block_size: int = 8, num_blocks: int = 32) -> PagedKVCache:
    cfg = ModelConfig(vocab_size=32, n_layers=2, d_model=32, n_heads=4, max_seq_len=128)
    return PagedKVCache(cfg, CacheConfig(block_size, num_blocks), device="cpu")


class TestAllocator:
    def test_round_trip(self) -> None:
        a = BlockAllocator(4)
        blocks = [a.allocate() for _ in range(4)]
        assert blocks == [3, 2, 1, 0]  # pops from the end, as the reference
        assert a.num_free == 0
        for b in blocks:
            a.free(b)
        assert a.num_free == 4
        a.check_invariants()

    def test_exhaustion_and_double_free(self) -> None:
        a = BlockAllocator(2)
        a.allocate_many(2)
        with pytest.raises(OutOfCacheMemory):
            a.allocate()
        with pytest.raises(OutOfCacheMemory):
            a.allocate_many(1)
        a.free(0)
        with pytest.raises(ValueError, match="double free"):
            a.free(0)

    def test_refcounts(self) -> None:
        a = BlockAllocator(2)
        b = a.allocate()
        a.incref(b)
        a.free(b)
        assert a.num_free == 1
        a.free(b)
        assert a.num_free == 2
        with pytest.raises(ValueError):
            a.incref(b)

    def test_allocate_many_matches_sequential_allocation(self) -> None:
        a, b = BlockAllocator(10), BlockAllocator(10)
        assert a.allocate_many(4) == [b.allocate() for _ in range(4)]


class TestCacheTables:
    def test_slots_follow_the_block_table(self) -> None:
        c = host_cache(block_size=4)
        slots = c.append(0, 6)
        blocks = c.tables[0].blocks
        assert slots == [blocks[p // 4] * 4 + p % 4 for p in range(6)]
        assert c.num_tokens(0) == 6

    def test_blocks_needed_is_exact(self) -> None:
        c = host_cache(block_size=8)
        assert c.blocks_needed(0, 1) == 1
        assert c.blocks_needed(0, 8) == 1
        assert c.blocks_needed(0, 9) == 2
        c.append(0, 5)
        assert c.blocks_needed(0, 3) == 0
        assert c.blocks_needed(0, 4) == 1

    def test_can_append_reports_exhaustion(self) -> None:
        c = host_cache(block_size=4, num_blocks=2)
        assert c.can_append(0, 8)
        assert not c.can_append(0, 9)

    def test_truncate_releases_tail_blocks(self) -> None:
        c = host_cache()
        total = c.num_free_blocks
        c.append(0, 24)
        assert c.num_free_blocks == total - 3
        c.truncate(0, 9)
        assert c.num_free_blocks == total - 2
        assert c.num_tokens(0) == 9
        c.allocator.check_invariants()

    def test_truncate_cannot_grow(self) -> None:
        c = host_cache()
        c.append(0, 4)
        with pytest.raises(ValueError, match="cannot grow"):
            c.truncate(0, 5)

    def test_append_after_truncate_reuses_the_partial_block(self) -> None:
        c = host_cache()
        c.append(0, 24)
        c.truncate(0, 9)
        before = c.tables[0].blocks
        slots = c.append(0, 3)
        assert c.num_tokens(0) == 12
        assert len(slots) == 3
        assert c.tables[0].blocks == before
        assert slots == [before[1] * 8 + p for p in (1, 2, 3)]

    def test_free_and_reset(self) -> None:
        c = host_cache()
        total = c.num_free_blocks
        c.append(0, 10)
        c.append(1, 3)
        c.free(999)  # unknown: no-op
        c.free(0)
        assert 0 not in c.tables
        c.reset()
        assert c.num_free_blocks == total
        assert c.tables == {}
        c.allocator.check_invariants()

    def test_append_many_is_all_or_nothing(self) -> None:
        c = host_cache(block_size=4, num_blocks=3)
        c.append(0, 4)
        with pytest.raises(OutOfCacheMemory):
            c.append_many([0, 1], [4, 8])  # 1 + 2 blocks, 2 free
        assert c.num_tokens(0) == 4
        assert c.num_free_blocks == 2

    def test_blocks_needed_many_predicts_append_many(self) -> None:
        rng = np.random.default_rng(1)
        c = host_cache(4, 256)
        ids = [5, 2, 9, 11]
        c.append(2, 3)
        for _ in range(8):
            counts = rng.integers(0, 9, len(ids))
            free = c.num_free_blocks
            need = c.blocks_needed_many(ids, counts)
            assert need == sum(c.blocks_needed(i, int(n)) for i, n in zip(ids, counts))
            c.append_many(ids, counts)
            assert free - c.num_free_blocks == need
            c.truncate_many(ids, [max(0, c.num_tokens(i) - int(rng.integers(0, 6))) for i in ids])

    def test_row_based_calls_match_id_based_calls(self) -> None:
        rng = np.random.default_rng(3)
        a, b = host_cache(4, 128), host_cache(4, 128)
        ids = [8, 3, 6, 1]
        a.append_many(ids, [1, 2, 3, 4])
        b.append_many(ids, [1, 2, 3, 4])
        rows = a.rows_if_all_present(ids)
        assert rows is not None and a.rows_if_all_present([8, 99]) is None
        assert 99 not in a.tables  # the probe created no row
        for _ in range(6):
            counts = rng.integers(0, 7, len(ids))
            assert a.blocks_needed_many(ids, counts, rows) == b.blocks_needed_many(ids, counts)
            assert a.append_many(ids, counts, rows).tolist() == b.append_many(ids, counts).tolist()
            assert np.array_equal(a.num_tokens_many(ids, rows), b.num_tokens_many(ids))
            ta, la, wa = a.table_rows(ids, rows)
            tb, lb, wb = b.table_rows(ids)
            assert wa == wb and np.array_equal(ta, tb) and np.array_equal(la, lb)
            keep = [max(0, b.num_tokens(i) - int(rng.integers(0, 5))) for i in ids]
            a.truncate_many(ids, keep, rows)
            b.truncate_many(ids, keep)
            assert a.tables == b.tables
        a.allocator.check_invariants()

    def test_generation_tracks_row_changes(self) -> None:
        c = host_cache(4, 64)
        g0 = c.generation
        c.append(1, 3)
        assert c.generation == g0 + 1
        c.append(1, 5)
        c.truncate(1, 2)
        assert c.generation == g0 + 1  # token counts do not move rows
        c.free(1)
        assert c.generation == g0 + 2
        c.append(2, 1)  # takes the freed row
        assert c.generation == g0 + 3

    def test_decoder_row_cache_follows_the_caches(self) -> None:
        from microserve_b200.speculative import SpeculativeDecoder

        tc, dc = host_cache(4, 64), host_cache(4, 64)
        dec = object.__new__(SpeculativeDecoder)
        dec.draft_cache = dc
        dec._row_cache = None
        ids = [4, 7]
        assert dec._rows_for(ids, tc) == (None, None)  # no rows yet: id-based calls
        for c in (tc, dc):
            c.append_many(ids, [2, 2])
        tr, dr = dec._rows_for(ids, tc)
        assert tr.tolist() == tc.rows_of(ids).tolist() and dr.tolist() == dc.rows_of(ids).tolist()
        assert dec._rows_for(list(ids), tc)[0] is tr  # same request list: kept
        tc.free(4)
        tc.append(9, 1)  # sequence 9 takes sequence 4's row
        tc.append(4, 2)
        tr2, _ = dec._rows_for(ids, tc)
        assert tr2.tolist() == tc.rows_of(ids).tolist() != tr.tolist()
        assert dec._rows_for([4, 4], tc) == (None, None)  # duplicates: append_many reports them

    def test_plan_blob_is_the_same_with_a_shared_config(self) -> None:
        import torch

        from microserve_b200.speculative import SpeculativeDecoder

        sc = SamplingConfig(temperature=0.7, top_p=0.8, max_new_tokens=100)
        blobs = []
        for configs in (None, [sc]):
            tc, dc = host_cache(4, 256), host_cache(4, 256)
            dec = object.__new__(SpeculativeDecoder)
            dec.gamma, dec.draft_cache, dec._row_cache = 3, dc, None
            reqs, gens = [], {}
            for i, n in enumerate([5, 9, 3]):
                r = Request(10 + i, list(range(n)), sc)
                r.rng_step = 4 + i
                reqs.append(r)
                gens[r.request_id] = torch.Generator().manual_seed(100 + i)
                tc.append(r.request_id, n - 1)
            plan = dec._plan(reqs, tc, gens, configs)
            dec._plan_draft(plan)
            blobs.append((plan.blob, plan.blob_d))
        assert np.array_equal(blobs[0][0], blobs[1][0])
        assert np.array_equal(blobs[0][1], blobs[1][1])

    def test_plan_without_a_generator_changes_nothing(self) -> None:
        import torch

        from microserve_b200.speculative import SpeculativeDecoder

        sc = SamplingConfig(temperature=0.7, max_new_tokens=100)
        tc, dc = host_cache(4, 256), host_cache(4, 256)
        dec = object.__new__(SpeculativeDecoder)
        dec.gamma, dec.draft_cache, dec._row_cache = 3, dc, None
        reqs = [Request(20 + i, list(range(6)), sc) for i in range(3)]
        for r in reqs:
            tc.append(r.request_id, 5)
            dc.append(r.request_id, 2)
        gens = {r.request_id: torch.Generator().manual_seed(1) for r in reqs[:2]}
        def state():
            return ({k: (c.tables[k].blocks, c.tables[k].num_tokens) for c in (tc, dc) for k in c.tables},
                    tc.num_free_blocks, dc.num_free_blocks)

        before = state()
        with pytest.raises(KeyError):
            dec._plan(reqs, tc, gens, [sc])
        assert state() == before

    def test_round_metadata_matches_a_per_request_construction(self) -> None:
        """The three blobs of one speculative round (draft pass 0, the later
        draft passes with the verify ids, the verify batch) against each
        request's values built one by one from the cache tables
        (reference speculative.py:115-155, :158-190 and batching.py:19-63)."""
        import torch

        from microserve_b200.speculative import SpeculativeDecoder

        G, bs = 3, 4
        sc = SamplingConfig(temperature=0.9, top_p=0.8, max_new_tokens=100)
        tc, dc = host_cache(bs, 256), host_cache(bs, 256)
        dec = object.__new__(SpeculativeDecoder)
        dec.gamma, dec.draft_cache, dec._row_cache = G, dc, None
        # (prompt length, generated tokens, target cached, draft cached)
        shapes = [(9, 0, 8, 8), (5, 3, 7, 6), (6, 2, 7, 7), (11, 1, 10, 3), (3, 4, 6, 5)]
        reqs, gens = [], {}
        for i, (lp, lo, tcd, dcd) in enumerate(shapes):
            r = Request(30 + i, [100 + 7 * i + k for k in range(lp)], sc)
            r.output_ids = [900 + 3 * i + k for k in range(lo)]
            r.rng_step = i
            reqs.append(r)
            gens[r.request_id] = torch.Generator().manual_seed(50 + i)
            tc.append(r.request_id, tcd)
            dc.append(r.request_id, dcd)
        dcached = [dc.num_tokens(r.request_id) for r in reqs]
        tcached = [tc.num_tokens(r.request_id) for r in reqs]
        plan = dec._plan(reqs, tc, gens, [sc])
        dec._plan_draft(plan)
        dec._plan_verify(plan, tc)

        def parts(blob_key: str, span_key: str) -> list[list[int]]:
            blob = getattr(plan, blob_key)
            return [blob[o : o + n].tolist() for o, n in getattr(plan, span_key)]

        a0 = parts("blob", "spans")
        ad = parts("blob_d", "spans_d")
        av = parts("blob_v", "spans_v")
        B = len(reqs)
        ids0, pos0, slots0, q0, ctx0, n0, dtab, rows0 = a0
        e = {k: [] for k in ("ids0", "pos0", "slots0", "q0", "ctx0", "n0", "rows0")}
        e["q0"].append(0)
        for r, dcd in zip(reqs, dcached):
            toks = r.prompt_ids + r.output_ids
            k = len(toks) - dcd
            e["ids0"] += toks[dcd:]
            e["pos0"] += list(range(dcd, dcd + k))
            e["slots0"] += [dc.tables[r.request_id].slot(p_, bs) for p_ in range(dcd, dcd + k)]
            e["q0"].append(e["q0"][-1] + k)
            e["ctx0"].append(dcd + k)
            e["n0"].append(k)
            e["rows0"].append(e["q0"][-1] - 1)
        assert (ids0, pos0, slots0, q0, ctx0, n0, rows0) == (
            e["ids0"], e["pos0"], e["slots0"], e["q0"], e["ctx0"], e["n0"], e["rows0"])
        width = len(dtab) // B
        for b, r in enumerate(reqs):
            blocks = dc.tables[r.request_id].blocks
            assert dtab[b * width : b * width + len(blocks)] == blocks
        # later draft passes: one token each, positions after the catch-up
        assert ad[1] == list(range(B + 1)) and ad[2] == [1] * B
        for j in range(1, G):
            pos, slots, ctx = ad[3 * j], ad[3 * j + 1], ad[3 * j + 2]
            want_pos = [dcd + k + j - 1 for dcd, k in zip(dcached, e["n0"])]
            assert pos == want_pos
            assert slots == [dc.tables[r.request_id].slot(p_, bs) for r, p_ in zip(reqs, want_pos)]
            assert ctx == [p_ + 1 for p_ in want_pos]
        # verify: uncomputed tokens then G proposal places per request
        idsv, scat = ad[3 * G], ad[3 * G + 1 :]
        posv, tslots, qv, ctxv, qlv, ttab, rowsv = av
        want_ids, want_pos, want_slots, want_q, want_scat = [], [], [], [0], [[] for _ in range(G)]
        for r, tcd in zip(reqs, tcached):
            toks = r.prompt_ids + r.output_ids
            npre = len(toks) - tcd
            base = want_q[-1]
            for j in range(G):
                want_scat[j].append(base + npre + j)
            want_ids += toks[tcd:] + [0] * G
            want_pos += list(range(tcd, tcd + npre + G))
            want_slots += [tc.tables[r.request_id].slot(p_, bs) for p_ in range(tcd, tcd + npre + G)]
            want_q.append(base + npre + G)
        assert idsv == want_ids and scat == want_scat
        assert posv == want_pos and tslots == want_slots and qv == want_q
        assert ctxv == [tcd + (q1 - q0_) for tcd, q0_, q1 in zip(tcached, want_q, want_q[1:])]
        assert qlv == [q1 - q0_ for q0_, q1 in zip(want_q, want_q[1:])]
        assert rowsv == [q - (G + 1) + i for q in want_q[1:] for i in range(G + 1)]
        wt = len(ttab) // B
        for b, r in enumerate(reqs):
            blocks = tc.tables[r.request_id].blocks
            assert ttab[b * wt : b * wt + len(blocks)] == blocks
        # sampling parameters: one entry per request, its generator's seed and its step
        from microserve_b200 import _lib

        o, n = plan.spans_d[0]
        params = np.frombuffer(plan.blob_d[o : o + n].tobytes(), dtype=_lib.SAMPLING_PARAMS_DTYPE)
        assert params["seed"].tolist() == [gens[r.request_id].initial_seed() for r in reqs]
        assert params["step"].tolist() == [r.rng_step for r in reqs]
        assert np.allclose(params["temperature"], 0.9) and np.allclose(params["top_p"], 0.8)

    def test_round_rollback_follows_the_reference(self) -> None:
        """After a round, the target keeps n_tokens + accepted, the draft
        min(its length, that), and each request gets its accepted prefix plus
        one token (reference speculative.py:191-226)."""
        import torch

        from microserve_b200.speculative import SpeculativeDecoder

        G, bs = 4, 4
        sc = SamplingConfig(temperature=0.7, max_new_tokens=100)
        tc, dc = host_cache(bs, 256), host_cache(bs, 256)
        dec = object.__new__(SpeculativeDecoder)
        dec.gamma, dec.draft_cache, dec._row_cache = G, dc, None
        dec.num_proposed = dec.num_accepted = 0
        reqs, gens = [], {}
        for i, lp in enumerate([7, 12, 5, 9]):
            r = Request(40 + i, list(range(lp)), sc)
            reqs.append(r)
            gens[r.request_id] = torch.Generator().manual_seed(i)
            tc.append(r.request_id, lp - 1)
            dc.append(r.request_id, lp - 1)
        n_tok = [len(r.prompt_ids) for r in reqs]
        plan = dec._plan(reqs, tc, gens, [sc])
        dec._plan_draft(plan)
        dec._plan_verify(plan, tc)
        d_len = [dc.num_tokens(r.request_id) for r in reqs]
        nacc = np.array([0, 4, 2, 1])
        tokens = np.arange(len(reqs) * (G + 1), dtype=np.int32).reshape(len(reqs), G + 1) + 500
        out = dec._finish(reqs, tc, plan, tokens, nacc)
        for b, r in enumerate(reqs):
            keep = n_tok[b] + int(nacc[b])
            assert out[b] == tokens[b, : nacc[b] + 1].tolist()
            assert tc.num_tokens(r.request_id) == keep == r.num_computed
            assert dc.num_tokens(r.request_id) == min(d_len[b], keep)
            assert len(tc.tables[r.request_id].blocks) == -(-keep // bs)
            assert (r.num_draft_proposed, r.num_draft_accepted, r.rng_step) == (G, nacc[b], 1)
        assert (dec.num_proposed, dec.num_accepted) == (G * len(reqs), int(nacc.sum()))
        tc.allocator.check_invariants()
        dc.allocator.check_invariants()

    def test_batched_truncate_and_append_change_nothing_on_error(self) -> None:
        c = host_cache(4, 64)
        c.append_many([1, 2, 3], [9, 5, 7])
        snap = ({k: (c.tables[k].blocks, c.tables[k].num_tokens) for k in c.tables},
                c.num_free_blocks)
        with pytest.raises(ValueError, match="cannot grow"):
            c.truncate_many([1, 2, 3], [4, 6, 2])  # sequence 2 would grow
        with pytest.raises(OutOfCacheMemory):
            c.append_many([1, 2, 3], [1, 1, 500])
        with pytest.raises(ValueError):
            c.truncate_many([1, 2], [3])
        assert ({k: (c.tables[k].blocks, c.tables[k].num_tokens) for k in c.tables},
                c.num_free_blocks) == snap
        c.allocator.check_invariants()

    def test_fork_shares_blocks(self) -> None:
        # reference tests/test_cache.py:159-183
        c = host_cache(4, 32)
        c.append(0, 16)
        free_before = c.num_free_blocks
        c.fork(0, 1)
        assert c.num_free_blocks == free_before
        assert c.tables[0].blocks == c.tables[1].blocks
        assert c.num_tokens(1) == 16
        for block in c.tables[0].blocks:
            assert c.allocator.refcount(block) == 2
        blocks = list(c.tables[1].blocks)
        c.free(0)
        for block in blocks:
            assert c.allocator.refcount(block) == 1
        c.free(1)
        c.allocator.check_invariants()
        c.append(0, 4)
        c.append(1, 4)
        with pytest.raises(ValueError, match="already exists"):
            c.fork(0, 1)

    def test_unshare_last_block_and_rollback_of_shared_blocks(self) -> None:
        c = host_cache(4, 32)
        c.append(0, 10)
        c.fork(0, 1)
        old_tail = c.tables[1].blocks[-1]
        c.unshare_last_block(1)
        assert c.tables[1].blocks[:-1] == c.tables[0].blocks[:-1]
        assert c.tables[1].blocks[-1] != old_tail
        assert c.allocator.refcount(old_tail) == 1
        c.unshare_last_block(1)  # already private: nothing changes
        assert c.allocator.refcount(c.tables[1].blocks[-1]) == 1
        # truncating both below the shared prefix releases each shared block once
        c.truncate_many([0, 1], [1, 1])
        assert c.allocator.refcount(c.tables[0].blocks[0]) == 2
        c.free(0)
        c.free(1)
        c.allocator.check_invariants()
        assert c.num_free_blocks == 32

    def test_vectorised_paths_match_single_calls(self) -> None:
        rng = np.random.default_rng(0)
        a, b = host_cache(4, 64), host_cache(4, 64)
        ids = [3, 1, 7]
        for _ in range(6):
            counts = rng.integers(1, 6, 3)
            got = a.append_many(ids, counts).tolist()
            want = [s for i, n in zip(ids, counts) for s in b.append(i, int(n))]
            assert got == want
            keep = [max(0, a.num_tokens(i) - int(rng.integers(0, 4))) for i in ids]
            a.truncate_many(ids, keep)
            for i, k in zip(ids, keep):
                b.truncate(i, k)
            assert a.tables == b.tables
        a.allocator.check_invariants()

    def test_table_rows_and_block_tables(self) -> None:
        c = host_cache(block_size=2)
        c.append(0, 5)
        c.append(1, 1)
        tables, lens = c.build_block_tables([0, 1])
        assert tables.shape == (2, 3)
        assert lens.tolist() == [5, 1]
        assert tables[1, 1:].tolist() == [0, 0]

    def test_tensor_methods_need_a_device(self) -> None:
        import torch

        c = host_cache()
        with pytest.raises(RuntimeError, match="CUDA"):
            c.write(0, torch.zeros(1, dtype=torch.long), torch.zeros(1, 4, 8), torch.zeros(1, 4, 8))


class TestScheduler:
    def _sched(self, **kw) -> tuple[Scheduler, PagedKVCache]:
        c = host_cache(block_size=4, num_blocks=kw.pop("num_blocks", 16))
        return Scheduler(SchedulerConfig(**kw), c), c

    def test_admission_never_over_commits(self) -> None:
        s, c = self._sched(max_batch_size=8, num_blocks=8)
        for i in range(6):
            s.add(Request(i, [1] * 9, SamplingConfig()))
        out = s.schedule(0.0)
        need = sum(c.blocks_needed(r.request_id, r.num_uncomputed) for r in out.scheduled)
        assert need <= c.num_free_blocks

    def test_fcfs_order_and_batch_cap(self) -> None:
        s, _ = self._sched(max_batch_size=2)
        for i, t in enumerate([3.0, 1.0, 2.0]):
            s.add(Request(i, [1, 2], SamplingConfig(), arrival_time=t))
        out = s.schedule(0.0)
        assert [r.request_id for r in out.scheduled] == [1, 2]

    def test_speculative_reservation(self) -> None:
        s, _ = self._sched(max_batch_size=4, num_blocks=4)
        s.tokens_per_step = 6
        for i in range(3):
            s.add(Request(i, [1], SamplingConfig()))
        out = s.schedule(0.0)
        # each request reserves ceil(6/4) = 2 blocks of the 4
        assert len(out.scheduled) == 2

    def test_preemption_frees_the_victim(self) -> None:
        s, c = self._sched(max_batch_size=4, num_blocks=4)
        reqs = [Request(i, [1] * 4, SamplingConfig(), arrival_time=float(i)) for i in range(2)]
        for r in reqs:
            s.add(r)
        out = s.schedule(0.0)
        for r in out.scheduled:
            c.append(r.request_id, r.num_uncomputed)
            r.num_computed = r.num_tokens
            r.output_ids.extend([1] * 8)  # each now needs 2 more blocks; 2 are free
        out = s.schedule(1.0)
        assert out.preempted and out.preempted[0].request_id == 1
        assert out.preempted[0].num_computed == 0
        assert c.num_tokens(1) == 0

    def test_request_tail(self) -> None:
        r = Request(0, [1, 2, 3], SamplingConfig(), output_ids=[4, 5])
        for s in range(6):
            assert r.tail(s) == r.all_ids[s:]


class TestConfig:
    def test_defaults_follow_the_reference(self) -> None:
        m = ModelConfig()
        assert m.d_ff == 352 and m.n_kv_heads == 4 and m.d_head == 32
        assert ModelConfig(d_model=64, n_heads=2).d_ff == 160
        assert SamplingConfig(temperature=0.0).greedy
        assert CacheConfig().num_slots == 16 * 512

    def test_validation(self) -> None:
        with pytest.raises(ValueError):
            ModelConfig(d_model=30, n_heads=4)
        with pytest.raises(ValueError):
            ModelConfig(n_heads=4, n_kv_heads=3)
        with pytest.raises(ValueError):
            SchedulerConfig(policy="nope")
        with pytest.raises(ValueError):
            ModelConfig(dtype="float16")

    def test_round_trip(self, tmp_path) -> None:
        cfg = EngineConfig(model=ModelConfig(n_kv_heads=2, dtype="bfloat16"),
                           speculative=SpeculativeConfig(enabled=True, gamma=3))
        p = tmp_path / "e.json"
        cfg.save(p)
        assert load_config(p) == cfg
        with pytest.raises(ValueError, match="unknown config key"):
            EngineConfig.from_dict({"bogus": 1})


def test_saved_checkpoint_loads_with_the_reference_config_class(tmp_path) -> None:
    """A checkpoint this package writes keeps ``config`` to the reference's
    ModelConfig fields (their names recorded from the reference by the fixture
    script), so ``ModelConfig(**payload["config"])`` of the reference
    (model.py:369-370) accepts it; the added fields come back on our side."""
    import dataclasses

    import torch

    from microserve_b200.config import ModelConfig
    from microserve_b200.model import checkpoint_payload, load_checkpoint

    with np.load(ROOT / "tests" / "golden" / "config_fixtures.npz") as z:
        ref_fields = [str(f) for f in z["ref/model_config_fields"]]
    cfg = ModelConfig(vocab_size=48, n_layers=1, d_model=32, n_heads=4, n_kv_heads=2,
                      dtype="bfloat16")
    embed = torch.randn(48, 32)
    state = {"embed.weight": embed, "lm_head.weight": embed, "norm.weight": torch.ones(32)}
    path = tmp_path / "ours.pt"
    torch.save(checkpoint_payload(cfg, state, {"step": 3}), path)
    payload = torch.load(path, weights_only=True)
    assert set(payload["config"]) == set(ref_fields)
    RefModelConfig = dataclasses.make_dataclass(  # the reference's field set, nothing more
        "RefModelConfig", [(f, object, dataclasses.field(default=None)) for f in ref_fields])
    RefModelConfig(**payload["config"])
    back, st = load_checkpoint(path)
    assert (back.n_kv_heads, back.dtype, back.d_model) == (2, "bfloat16", 32)
    assert st["lm_head.weight"].data_ptr() == st["embed.weight"].data_ptr()  # one storage


def test_checkpoint_in_the_reference_format_loads(tmp_path) -> None:
    """A payload laid out as the reference's Transformer.save writes it
    (reference model.py:356-362): config keys of the reference only, a
    float32 state dict and extra entries."""
    import torch

    from microserve_b200.model import load_checkpoint

    ref_cfg = dict(vocab_size=65, n_layers=2, d_model=64, n_heads=4, d_ff=176, max_seq_len=256,
                   rope_theta=10000.0, norm_eps=1e-5, tie_weights=True, dropout=0.0)
    state = {"embed.weight": torch.randn(65, 64), "norm.weight": torch.ones(64)}
    path = tmp_path / "draft.pt"
    torch.save({"config": ref_cfg, "state_dict": state, "step": 1200, "val_loss": 1.52}, path)
    cfg, got = load_checkpoint(path)
    assert (cfg.d_ff, cfg.n_kv_heads, cfg.dtype, cfg.d_head) == (176, 4, "float32", 16)
    assert torch.equal(got["embed.weight"], state["embed.weight"])
    cfg16, _ = load_checkpoint(path, dtype="bfloat16")
    assert cfg16.dtype == "bfloat16"
    # anything but plain values and tensors is refused
    torch.save({"config": ref_cfg, "state_dict": state, "obj": object()}, tmp_path / "bad.pt")
    with pytest.raises(Exception):
        load_checkpoint(tmp_path / "bad.pt")


@pytest.mark.parametrize("case", range(5))
def test_scheduler_decisions_match_the_reference(case: int) -> None:
    """The same synthetic serving run under memory pressure, driven through
    the reference's Scheduler by ``make_golden.py`` and through this one:
    every step schedules and preempts the same requests in the same order
    (FCFS / SJF / LIFO, continuous and static batching, speculative
    reservations of 4 and 6 slots)."""
    import sys

    sys.path.insert(0, str(ROOT / "tests" / "golden"))
    import workloads as wl

    spec = wl.SCHEDULER_CASES[case]
    cache = host_cache(block_size=4, num_blocks=spec[3])
    trace = wl.scheduler_trace(Request, Scheduler, SamplingConfig, SchedulerConfig, cache, spec)
    with np.load(ROOT / "tests" / "golden" / "config_fixtures.npz") as z:
        want = z[f"sched/{case}"].tolist()
        steps = int(z[f"sched/{case}/steps"])
    assert len(trace) == steps
    assert [x for rec in trace for x in rec] == want


def test_chunked_prefill_charges_only_the_next_chunk() -> None:
    """With prefill_chunk the token budget and the block demand count the
    chunk a prefilling request processes next, not its whole prompt."""
    cache = host_cache(block_size=4, num_blocks=64)
    s = Scheduler(SchedulerConfig(max_batch_size=8, max_batched_tokens=40, prefill_chunk=16),
                  cache)
    for i in range(4):
        s.add(Request(i, [1] * 30, SamplingConfig()))
    out = s.schedule(0.0)
    # 16 + 16 fit the 40-token budget, a third chunk does not
    assert [r.request_id for r in out.scheduled] == [0, 1]
    assert [s.step_len(r) for r in out.scheduled] == [16, 16]
    plain = Scheduler(SchedulerConfig(max_batch_size=8, max_batched_tokens=40),
                      host_cache(block_size=4, num_blocks=64))
    for i in range(4):
        plain.add(Request(i, [1] * 30, SamplingConfig()))
    assert [r.request_id for r in plain.schedule(0.0).scheduled] == [0]
    with pytest.raises(ValueError):
        SchedulerConfig(prefill_chunk=0)


def test_reserved_capacity_and_lazy_truncation() -> None:
    """reserve_many gives blocks without tokens; appends inside the reserve
    take no block and land on the reserved blocks; truncate with keep_blocks
    keeps them; free returns everything."""
    c = host_cache(block_size=4, num_blocks=32)
    c.append_many([0, 1], [5, 2])
    free0 = c.num_free_blocks
    assert c.reserve_many([0, 1], [13, 3])  # 4 blocks for seq 0 (had 2), 1 for seq 1 (had 1)
    assert c.num_free_blocks == free0 - 2 and c.num_tokens(0) == 5
    table0 = list(c.tables[0].blocks)
    slots = c.append_many([0], [6]).tolist()  # positions 5..10, inside the reserve
    assert c.num_free_blocks == free0 - 2
    assert slots == [table0[p // 4] * 4 + p % 4 for p in range(5, 11)]
    c.truncate_many([0], [6], keep_blocks=True)
    assert c.num_tokens(0) == 6 and list(c.tables[0].blocks) == table0
    assert not c.reserve_many([1], [4 * 40])  # more than the pool: nothing changes
    assert c.num_free_blocks == free0 - 2
    with pytest.raises(ValueError):
        c.truncate_many([0], [9], keep_blocks=True)
    c.free(0)
    c.free(1)
    assert c.num_free_blocks == 32
    c.allocator.check_invariants()
