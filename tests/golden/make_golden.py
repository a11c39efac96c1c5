"""Generate the golden fixtures by running the unmodified MicroServe reference.

Run in a container that has the reference source tree:

    python tests/golden/make_golden.py /path/to/microserve

It imports ``microserve`` from ``<root>/src`` and writes small ``.npz`` files
next to this script.  The tests only read the ``.npz`` files (the reference
is not needed at test time).  Every fixture records the reference call it
came from.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


def state_arrays(model: torch.nn.Module, prefix: str) -> dict[str, np.ndarray]:
    return {prefix + k: v.detach().cpu().numpy().astype(np.float32)
            for k, v in model.state_dict().items()}


def main(ref_root: str) -> None:
    sys.path.insert(0, str(Path(ref_root) / "src"))
    from microserve.batching import build_paged_batch
    from microserve.cache import PagedKVCache
    from microserve.config import (CacheConfig, EngineConfig, ModelConfig, SamplingConfig,
                                   SchedulerConfig, SpeculativeConfig)
    from microserve.engine import LLMEngine
    from microserve.model import Transformer
    from microserve.sampling import probs_from_logits
    from microserve.speculative import SpeculativeDecoder, verify_proposals

    torch.set_num_threads(1)

    def make_model(cfg: ModelConfig, seed: int, amplify: float) -> Transformer:
        # the reference test fixture recipe (tests/conftest.py:41-56)
        torch.manual_seed(seed)
        m = Transformer(cfg).eval()
        with torch.no_grad():
            for blk in m.blocks:
                blk.attn.o_proj.weight *= amplify
                blk.ffn.down_proj.weight *= amplify
        return m

    def dense_greedy(model: Transformer, prompt: list[int], n: int) -> list[int]:
        # tests/conftest.py:74-85
        past = None
        cur = torch.tensor(prompt)[None]
        out = []
        for _ in range(n):
            with torch.no_grad():
                logits, past = model(cur, past_kv=past, return_cache=True)
            tok = int(logits[0, -1].argmax())
            out.append(tok)
            cur = torch.tensor([[tok]])
        return out

    tcfg = ModelConfig(vocab_size=32, n_layers=2, d_model=32, n_heads=4, max_seq_len=128)
    dcfg = ModelConfig(vocab_size=32, n_layers=1, d_model=16, n_heads=2, max_seq_len=128)
    target = make_model(tcfg, 0, 20.0)
    draft = make_model(dcfg, 1, 20.0)
    out: dict[str, np.ndarray] = {}
    out.update(state_arrays(target, "target/"))
    out.update(state_arrays(draft, "draft/"))
    out["target_cfg"] = np.array([32, 2, 32, 4, 4, int(tcfg.d_ff), 128])
    out["draft_cfg"] = np.array([32, 1, 16, 2, 2, int(dcfg.d_ff), 128])

    # -- paged forward logits (model.py:339 forward_paged via batching.py:19) --
    gen = torch.Generator().manual_seed(7)
    rnd = lambda n: torch.randint(0, 32, (n,), generator=gen).tolist()  # noqa: E731
    cases = {
        "prefill11": ([rnd(11)], None),
        "unequal": ([rnd(n) for n in (3, 9, 16, 1)], None),
    }
    for name, (seqs, _) in cases.items():
        cache = PagedKVCache(tcfg, CacheConfig(block_size=8, num_blocks=32))
        batch = build_paged_batch(cache, list(range(len(seqs))), seqs, [0] * len(seqs))
        with torch.no_grad():
            logits = target.forward_paged(batch, cache)
        out[f"fwd/{name}/tokens"] = np.concatenate([np.asarray(s) for s in seqs])
        out[f"fwd/{name}/lens"] = np.asarray([len(s) for s in seqs])
        out[f"fwd/{name}/logits"] = logits.numpy()
    # decode after prefill, with a mixed prefill+decode pass (test_model.py:145-162)
    a, b = rnd(7), rnd(5)
    tok = rnd(1)
    cache = PagedKVCache(tcfg, CacheConfig(block_size=8, num_blocks=32))
    build = lambda ids, toks, st: build_paged_batch(cache, ids, toks, st)  # noqa: E731
    with torch.no_grad():
        target.forward_paged(build([0], [a], [0]), cache)
        mixed = target.forward_paged(build([0, 1], [tok, b], [7, 0]), cache)
    out["fwd/mixed/a"] = np.asarray(a)
    out["fwd/mixed/b"] = np.asarray(b)
    out["fwd/mixed/tok"] = np.asarray(tok)
    out["fwd/mixed/logits"] = mixed.numpy()

    # -- greedy streams: dense reference and SpeculativeDecoder.generate --
    prompts = [rnd(6), rnd(11), rnd(3)]
    for i, p in enumerate(prompts):
        out[f"greedy/{i}/prompt"] = np.asarray(p)
        out[f"greedy/{i}/dense"] = np.asarray(dense_greedy(target, p, 20))
        for gamma in (1, 2, 3, 5):
            dec = SpeculativeDecoder(target, draft, CacheConfig(block_size=8, num_blocks=32),
                                     gamma=gamma)
            got = dec.generate(p, SamplingConfig(temperature=0.0, max_new_tokens=20))
            out[f"greedy/{i}/spec{gamma}"] = np.asarray(got)
            out[f"greedy/{i}/spec{gamma}_counts"] = np.asarray([dec.num_accepted, dec.num_proposed])

    # -- engine greedy (test_speculative.py:211-245 shape) --
    eprompts = [rnd(n) for n in (4, 9, 6)]
    for gamma in (1, 3, 5):
        cfg = EngineConfig(model=tcfg, cache=CacheConfig(block_size=8, num_blocks=128),
                           scheduler=SchedulerConfig(max_batch_size=3),
                           speculative=SpeculativeConfig(enabled=True, gamma=gamma))
        eng = LLMEngine(target, cfg, draft_model=draft)
        reqs = [eng.add_request(p, SamplingConfig(temperature=0.0, max_new_tokens=16))
                for p in eprompts]
        outs = {o.request_id: o.output_ids for o in eng.run()}
        for j, r in enumerate(reqs):
            out[f"engine/g{gamma}/{j}"] = np.asarray(outs[r.request_id])
        out[f"engine/g{gamma}/counts"] = np.asarray(
            [eng.stats.num_draft_accepted, eng.stats.num_draft_proposed])
    for j, p in enumerate(eprompts):
        out[f"engine/prompt/{j}"] = np.asarray(p)

    # -- sampling filters (sampling.py:54-74 probs_from_logits) --
    g2 = torch.Generator().manual_seed(11)
    settings = [(0.8, None, None), (1.0, 5, None), (1.0, None, 0.9), (0.7, 5, 0.9),
                (1.3, None, 0.5), (1.0, 50, 0.9), (0.0, None, None)]
    for vocab in (32, 1000):
        logits = torch.randn(6, vocab, generator=g2) * 2.0
        out[f"filter/v{vocab}/logits"] = logits.numpy()
        for si, (t, k, p) in enumerate(settings):
            probs = probs_from_logits(logits, SamplingConfig(temperature=t, top_k=k, top_p=p))
            out[f"filter/v{vocab}/s{si}"] = probs.numpy()
    out["filter/settings"] = np.asarray(
        [[t, -1 if k is None else k, -1.0 if p is None else p] for t, k, p in settings])

    # -- verify_proposals deterministic cases (test_speculative.py:36-61) --
    r1 = verify_proposals(torch.tensor([[0.5, 0.5]]), torch.tensor([[1.0, 0.0], [1.0, 0.0]]), [0],
                          torch.Generator().manual_seed(0))
    r2 = verify_proposals(torch.tensor([[0.0, 1.0]]), torch.tensor([[1.0, 0.0], [1.0, 0.0]]), [1],
                          torch.Generator().manual_seed(0))
    out["verify/dominates"] = np.asarray([r1.num_accepted, *r1.tokens])
    out["verify/impossible"] = np.asarray([r2.num_accepted, *r2.tokens])

    # -- GQA pin: a grouped model equals the reference MHA model with each
    # kv head's rows repeated per group --
    gcfg = ModelConfig(vocab_size=48, n_layers=2, d_model=64, n_heads=8, max_seq_len=64)
    torch.manual_seed(3)
    mha = Transformer(gcfg).eval()
    hkv, dh, group = 2, 8, 4
    gqa_state = {}
    with torch.no_grad():
        for i, blk in enumerate(mha.blocks):
            for nm in ("k_proj", "v_proj"):
                w = getattr(blk.attn, nm).weight
                small = torch.randn(hkv * dh, 64) * 0.3
                gqa_state[f"blocks.{i}.attn.{nm}.weight"] = small.numpy()
                w.copy_(small.view(hkv, dh, 64).repeat_interleave(group, 0).reshape(64, 64))
            blk.attn.o_proj.weight *= 10
            blk.ffn.down_proj.weight *= 10
    for k, v in mha.state_dict().items():
        if k not in gqa_state:
            gqa_state[k] = v.numpy().astype(np.float32)
    seq = torch.randint(0, 48, (13,), generator=gen).tolist()
    with torch.no_grad():
        dense, _ = mha(torch.tensor(seq)[None])
    for k, v in gqa_state.items():
        out["gqa/" + k] = v
    out["gqa/tokens"] = np.asarray(seq)
    out["gqa/logits"] = dense[0].numpy()

    np.savez_compressed(HERE / "reference_fixtures.npz", **out)
    print(f"wrote {HERE / 'reference_fixtures.npz'} with {len(out)} arrays")


def _ref_model(shape, state: dict[str, np.ndarray]):
    """The reference's Transformer with the given float32 weights."""
    from microserve.config import ModelConfig
    from microserve.model import Transformer

    cfg = ModelConfig(vocab_size=shape.vocab_size, n_layers=shape.n_layers,
                      d_model=shape.d_model, n_heads=shape.n_heads, d_ff=shape.d_ff,
                      max_seq_len=shape.max_seq_len, rope_theta=shape.rope_theta)
    m = Transformer(cfg).eval()
    m.load_state_dict({k: torch.from_numpy(np.ascontiguousarray(v)) for k, v in state.items()})
    return m


def _run_engine(target, draft, gamma: int, prompts, budgets, cache_blocks: int,
                max_batch: int, max_tokens: int,
                preemptions: bool = False) -> tuple[list[list[int]], list[int]]:
    """LLMEngine.run of the reference (engine.py:155-202) at temperature 0;
    counts are [accepted, proposed, steps] (+ preemptions when asked)."""
    from microserve.config import (CacheConfig, EngineConfig, SamplingConfig, SchedulerConfig,
                                   SpeculativeConfig)
    from microserve.engine import LLMEngine

    cfg = EngineConfig(model=target.cfg, cache=CacheConfig(block_size=16, num_blocks=cache_blocks),
                       scheduler=SchedulerConfig(max_batch_size=max_batch,
                                                 max_batched_tokens=max_tokens),
                       speculative=SpeculativeConfig(enabled=True, gamma=gamma))
    eng = LLMEngine(target, cfg, draft_model=draft)
    reqs = [eng.add_request(p, SamplingConfig(temperature=0.0, max_new_tokens=int(b)))
            for p, b in zip(prompts, budgets, strict=True)]
    outs = {o.request_id: o.output_ids for o in eng.run()}
    counts = [eng.stats.num_draft_accepted, eng.stats.num_draft_proposed, eng.stats.num_steps]
    if preemptions:
        counts.append(eng.stats.num_preemptions)
    return [outs[r.request_id] for r in reqs], counts


def config_fixtures() -> None:
    """Token streams of the reference engine on the character-level configurations
    (config 0: 8 requests, gamma 3; config 2: a 64-request subset of the
    continuous-batching workload at gamma 1/2/3/5, and 24 requests of it in a
    64-block pool where the scheduler preempts between speculative rounds),
    greedy, random-init weights from ``workloads.init_state``; the reference
    ModelConfig's field names; top-p tie choices; the scheduler's decisions
    under memory pressure."""
    import dataclasses

    from microserve.config import CacheConfig, ModelConfig

    import workloads as wl

    torch.set_num_threads(1)
    out: dict[str, np.ndarray] = {}
    out["ref/model_config_fields"] = np.asarray([f.name for f in dataclasses.fields(ModelConfig)])
    for amp in (1.0, 20.0):
        tag = f"a{int(amp)}"
        target = _ref_model(wl.CHAR_TARGET, wl.init_state(wl.CHAR_TARGET, 0, amp))
        draft = _ref_model(wl.CHAR_DRAFT, wl.init_state(wl.CHAR_DRAFT, 1, amp))
        w0 = wl.config0()
        toks, counts = _run_engine(target, draft, 3, w0.prompts, w0.max_new_tokens, 256, 8, 2048)
        for j, t in enumerate(toks):
            out[f"cfg0/{tag}/g3/{j}"] = np.asarray(t)
        out[f"cfg0/{tag}/g3/counts"] = np.asarray(counts)
        w2 = wl.config2(64)
        for gamma in ((1, 2, 3, 5) if amp == 1.0 else (3,)):
            toks, counts = _run_engine(target, draft, gamma, w2.prompts, w2.max_new_tokens, 4096,
                                       64, 64 * 600)
            for j, t in enumerate(toks):
                out[f"cfg2/{tag}/g{gamma}/{j}"] = np.asarray(t)
            out[f"cfg2/{tag}/g{gamma}/counts"] = np.asarray(counts)
            print(f"config 2 amplify {amp} gamma {gamma}: counts {counts}")
    # the same workload under memory pressure: 24 requests in 64 blocks of 16,
    # so the scheduler preempts running requests between speculative rounds
    # and recomputes them by prefill (scheduler.py:196-225, engine.py:163-166)
    wp = wl.config2(24, seed=5)
    for amp in (1.0, 20.0):
        tag = f"a{int(amp)}"
        target = _ref_model(wl.CHAR_TARGET, wl.init_state(wl.CHAR_TARGET, 0, amp))
        draft = _ref_model(wl.CHAR_DRAFT, wl.init_state(wl.CHAR_DRAFT, 1, amp))
        toks, counts = _run_engine(target, draft, 3, wp.prompts, wp.max_new_tokens, 64, 24, 4096,
                                   preemptions=True)
        for j, t in enumerate(toks):
            out[f"cfg2p/{tag}/g3/{j}"] = np.asarray(t)
        out[f"cfg2p/{tag}/g3/counts"] = np.asarray(counts)
        print(f"config 2 amplify {amp} under memory pressure: counts {counts}")
    # top-p with exact ties at the cut (sampling.py:34-51): which tied tokens
    # survive follows torch.sort's order among equal values, which is not
    # stable for long rows
    from microserve.sampling import apply_top_p

    x = torch.zeros(1, 40000)
    x[0, ::3] = 1.0
    out["ties/long_row_kept"] = torch.isfinite(apply_top_p(x.clone(), 0.3)[0]).nonzero().flatten().numpy()
    x = torch.tensor([[2.0, 1.0, 1.0, 1.0, 1.0, 1.0, 0.0, 1.0]])
    out["ties/short_row_kept"] = torch.isfinite(apply_top_p(x.clone(), 0.5)[0]).nonzero().flatten().numpy()

    # scheduler decisions under memory pressure (scheduler.py:173-258)
    from microserve.cache import PagedKVCache
    from microserve.config import SamplingConfig, SchedulerConfig
    from microserve.scheduler import Request, Scheduler

    for ci, case in enumerate(wl.SCHEDULER_CASES):
        cache = PagedKVCache(ModelConfig(vocab_size=50, n_layers=1, d_model=8, n_heads=2),
                             CacheConfig(block_size=4, num_blocks=case[3]))
        trace = wl.scheduler_trace(Request, Scheduler, SamplingConfig, SchedulerConfig, cache, case)
        out[f"sched/{ci}"] = np.concatenate([np.asarray(r, dtype=np.int64) for r in trace])
        out[f"sched/{ci}/steps"] = np.asarray(len(trace))
        print(f"scheduler case {case}: {len(trace)} steps, "
              f"{trace[-1][-1]} preemptions")
    np.savez_compressed(HERE / "config_fixtures.npz", **out)
    print(f"wrote {HERE / 'config_fixtures.npz'} with {len(out)} arrays")


def kat_fixtures(ref_root: Path) -> None:
    """The trained-weight known answer: the reference's own checkpoints
    (artifacts/target.pt, draft.pt, loaded with weights_only=True), the eight
    32-token prompts of scripts/verify_speculative.py:236-241 (seed 20240) as
    token ids, the dense greedy continuations (48 tokens) and, per gamma in
    1/2/4/7, the speculative outputs and acceptance counts per prompt.  The
    published acceptance rates (artifacts/spec_stats.json:6-35) are the last
    prompt's, because the script resets the decoder before each prompt; they
    are checked here and stored."""
    import json

    from microserve.config import CacheConfig, SamplingConfig
    from microserve.data import load_corpus, sample_prompts
    from microserve.model import Transformer
    from microserve.speculative import SpeculativeDecoder
    from microserve.tokenizer import CharTokenizer

    torch.set_num_threads(1)
    seed = 20240
    torch.manual_seed(seed)
    art = ref_root / "artifacts"
    out: dict[str, np.ndarray] = {}
    models = {}
    for name in ("target", "draft"):
        payload = torch.load(art / f"{name}.pt", map_location="cpu", weights_only=True)
        c = payload["config"]
        out[f"{name}_cfg"] = np.asarray([c["vocab_size"], c["n_layers"], c["d_model"],
                                         c["n_heads"], c["n_heads"], c["d_ff"], c["max_seq_len"]])
        for k, v in payload["state_dict"].items():
            if k != "lm_head.weight":  # tied: the same tensor as embed.weight
                out[f"{name}/{k}"] = v.float().numpy()
        models[name] = Transformer.from_checkpoint(art / f"{name}.pt")
    tok = CharTokenizer.from_file(art / "tokenizer.json")
    corpus = load_corpus(ref_root / "data" / "tinyshakespeare.txt", tokenizer=tok)
    gen = torch.Generator().manual_seed(seed)
    prompts = sample_prompts(corpus, 8, [32] * 8, gen)
    target, draft = models["target"], models["draft"]
    dense = [dense_greedy_ref(target, p, 48) for p in prompts]
    out["prompts"] = np.asarray(prompts)
    out["dense"] = np.asarray(dense)
    stats = json.loads((art / "spec_stats.json").read_text())["greedy_equivalence"]
    published = {r["gamma"]: r["acceptance_rate"] for r in stats}
    cache_cfg = CacheConfig(block_size=16, num_blocks=256)
    for gamma in (1, 2, 4, 7):
        dec = SpeculativeDecoder(target, draft, cache_cfg, gamma=gamma)
        counts = []
        for i, p in enumerate(prompts):
            dec.reset()
            got = dec.generate(p, SamplingConfig(temperature=0.0, max_new_tokens=48), seq_id=i)
            assert got == dense[i], (gamma, i)
            out[f"spec{gamma}/{i}"] = np.asarray(got)
            counts.append([dec.num_accepted, dec.num_proposed])
        out[f"spec{gamma}/counts"] = np.asarray(counts)
        last = counts[-1][0] / counts[-1][1]
        assert abs(last - published[gamma]) < 1e-12, (gamma, last, published[gamma])
        out[f"spec{gamma}/published_acceptance"] = np.asarray(published[gamma])
        print(f"KAT gamma {gamma}: acceptance {last:.7f} (published {published[gamma]:.7f})")
    np.savez_compressed(HERE / "kat_fixtures.npz", **out)
    print(f"wrote {HERE / 'kat_fixtures.npz'} with {len(out)} arrays")


def dense_greedy_ref(model, prompt: list[int], n: int) -> list[int]:
    """Greedy continuation through the reference's dense path (its
    scripts/verify_speculative.py:49-60 procedure)."""
    past = None
    cur = torch.tensor(prompt)[None]
    out = []
    for _ in range(n):
        with torch.no_grad():
            logits, past = model(cur, past_kv=past, return_cache=True)
        t = int(logits[0, -1].argmax())
        out.append(t)
        cur = torch.tensor([[t]])
    return out


if __name__ == "__main__":
    import argparse

    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("reference_root", help="the MicroServe source tree (contains src/, artifacts/)")
    ap.add_argument("--only", choices=["tiny", "configs", "kat"], default=None)
    args = ap.parse_args()
    root = Path(args.reference_root)
    sys.path.insert(0, str(root / "src"))
    sys.path.insert(0, str(HERE))
    if args.only in (None, "tiny"):
        main(str(root))
    if args.only in (None, "configs"):
        config_fixtures()
    if args.only in (None, "kat"):
        kat_fixtures(root)
