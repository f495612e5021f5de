"""Generate the golden fixtures in this folder by running the REFERENCE itself (actkv-open's torch
path) on seeded inputs from tests/cases.py.

Run in a container that has the reference checked out (it is not needed anywhere else):

    ACTKV_REFERENCE=/path/to/actkv-open python tests/golden/make_golden.py

Triton is blocked before the reference is imported, so its dispatchers take the pure torch code
(actkv/kernels/lse_attn.py:143-144, actkv/kernels/compaction.py:99-100): that torch code is the
reference behaviour the fixtures record.  Each fixture is an .npz of inputs and outputs; large
inputs (BASELINE config 1's cache) are rebuilt from their seed by tests/cases.py and checked
against the sha256 stored here.
"""
from __future__ import annotations

import json
import math
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))          # tests/ (for cases.py)
sys.modules["triton"] = None                       # force the reference's torch path
sys.dont_write_bytecode = True
REF = os.environ.get("ACTKV_REFERENCE")
if not REF or not os.path.isdir(os.path.join(REF, "actkv")):
    raise SystemExit("set ACTKV_REFERENCE to a checkout of actkv-open (the folder holding actkv/)")
sys.path.insert(0, REF)

import cases  # noqa: E402
from actkv.config import EvictionConfig  # noqa: E402
from actkv.eviction import ActionLRFU, reduce_heads, top_p_mask  # noqa: E402
from actkv.kernels import compaction as ref_compaction  # noqa: E402
from actkv.kernels import lse_attn as ref_lse  # noqa: E402
from actkv.paged import PagedKVCache, keep_mask_from_scores  # noqa: E402

assert not ref_lse.HAS_TRITON and not ref_compaction.HAS_TRITON


def save(name, **arrays):
    meta = arrays.pop("meta", {})
    arrays = {k: (v.numpy() if isinstance(v, torch.Tensor) else np.asarray(v)) for k, v in arrays.items()}
    np.savez_compressed(os.path.join(HERE, name), meta=np.array(json.dumps(meta)), **arrays)
    print("wrote", name, sum(a.nbytes for a in arrays.values()), "bytes raw")


def ref_cache(case: cases.SessionCase) -> PagedKVCache:
    c = PagedKVCache(case.num_blocks, case.bs, case.hkv, case.d, n_layers=case.n_layers,
                     dtype=cases.DTYPES[case.dtype], device="cpu")
    c.kv.copy_(case.kv)
    c.free = list(case.free)
    for r, (t, n) in enumerate(zip(case.tables, case.seq_lens)):
        c.tables[r] = list(t)
        c.seq_used[r] = n
    return c


# --------------------------------------------------------------------------- scoring (A = 1 steps)
def gen_scores():
    shapes = [([37], 4, 2, 32, 16), ([5, 64, 100], 8, 2, 64, 16), ([33, 17], 6, 3, 24, 8),
              ([50], 1, 1, 16, 16), ([129, 16, 1], 16, 4, 128, 16)]
    out = {}
    for i, (lens, hq, hkv, d, bs) in enumerate(shapes):
        case = cases.build_sessions(100 + i, 1, hq, hkv, d, bs, lens, [3] * len(lens))
        cache = ref_cache(case)
        reqs = list(range(len(lens)))
        bt, seq = cache.block_table(reqs), cache.seq_tensor(reqs)
        width = bt.shape[1] * bs
        o = torch.zeros(len(reqs), hkv, width)
        ns = torch.zeros(len(reqs), dtype=torch.int32)
        qs, lses = [], []
        for step in range(3):
            q = torch.stack([case.q[r][0, step] for r in reqs])        # [R, Hq, D]
            _, lse = ref_lse.paged_decode_attention_ref(q, cache.kv[0], bt, seq)
            ref_lse.action_scores(q, cache.kv[0], bt, seq, lse, o, ns)
            qs.append(q)
            lses.append(lse)
        p = f"c{i}_"
        out.update({p + "kv_sha": np.array(cases.digest(cache.kv)), p + "bt": bt, p + "seq": seq, p + "q": torch.stack(qs),
                    p + "lse": torch.stack(lses), p + "out": o, p + "n_seen": ns})
    save("scores_small.npz", meta={"n": len(shapes), "shapes": shapes}, **out)


# --------------------------------------------------------------------------- compaction plans
def adversarial_masks(n, bs, g):
    m = {}
    m["alternating"] = torch.arange(n) % 2 == 0
    m["all_keep"] = torch.ones(n, dtype=torch.bool)
    m["sinks_only"] = torch.arange(n) < 4
    one = torch.zeros(n, dtype=torch.bool)
    one[torch.arange(0, n, bs)] = True
    m["one_per_block"] = one
    m["none"] = torch.zeros(n, dtype=torch.bool)
    tail = torch.zeros(n, dtype=torch.bool)
    tail[n // 2:] = True
    m["tail_half"] = tail
    r = torch.zeros(n, dtype=torch.bool)
    r[torch.randperm(n, generator=g)[: n // 3]] = True
    m["random_third"] = r
    return m


def gen_plans():
    g = torch.Generator().manual_seed(5)
    out, names = {}, []
    params = [(100, 40, 16), (17, 10, 16), (64, 64, 16), (200, 3, 8), (1, 1, 16), (4096, 409, 16),
              (33, 0, 16)]
    for i, (n, budget, bs) in enumerate(params):
        keep = torch.zeros(n, dtype=torch.bool)
        keep[torch.randperm(n, generator=g)[:budget]] = True
        masks = {"random": keep, **adversarial_masks(n, bs, g)}
        table = torch.randperm(math.ceil(n / bs) + 4, generator=g)
        for mname, m in masks.items():
            plan = ref_compaction.plan_compaction(m, n, table, bs)
            key = f"p{len(names)}_"
            names.append([n, bs, mname])
            out.update({key + "keep": m, key + "table": table, key + "src": plan.src_slots,
                        key + "dst": plan.dst_slots, key + "perm": plan.perm,
                        key + "drop": np.int64(plan.drop_blocks)})
    save("plans.npz", meta={"cases": names}, **out)


# --------------------------------------------------------------------------- cache compaction
def gen_compact():
    out, names = {}, []
    g = torch.Generator().manual_seed(9)
    for i, (lens, budget_frac, layers, bs) in enumerate([([150], 0.4, 2, 16), ([40], 0.97, 2, 16),
                                                         ([33, 70, 5], 0.5, 2, 16), ([200, 64], 0.2, 3, 8)]):
        case = cases.build_sessions(300 + i, layers, 4, 2, 32, bs, lens, [1] * len(lens))
        cache = ref_cache(case)
        kv0 = cache.kv.clone()
        keeps, perms = [], []
        for r, n in enumerate(lens):
            keep = torch.zeros(n, dtype=torch.bool)
            keep[torch.randperm(n, generator=g)[: max(1, int(budget_frac * n))]] = True
            keeps.append(keep)
            perms.append(cache.compact(r, keep))
        key = f"m{i}_"
        names.append(lens)
        out[key + "kv0_sha"] = np.array(cases.digest(kv0))
        out[key + "kv1_sha"] = np.array(cases.digest(cache.kv))
        out[key + "free0"] = np.asarray(case.free, np.int64)
        out[key + "free1"] = np.asarray(cache.free, np.int64)
        for r in range(len(lens)):
            out[key + f"table0_{r}"] = np.asarray(case.tables[r], np.int64)
            out[key + f"table1_{r}"] = np.asarray(cache.tables[r], np.int64)
            out[key + f"keep_{r}"] = keeps[r]
            out[key + f"perm_{r}"] = perms[r]
            out[key + f"seq1_{r}"] = np.int64(cache.seq_used[r])
    save("compact.npz", meta={"cases": names}, **out)


# --------------------------------------------------------------------------- keep masks
def gen_keep_masks():
    g = torch.Generator().manual_seed(11)
    out, names = {}, []
    shapes = [(40,), (3, 40), (2, 3, 40), (36, 8, 300), (5, 1000), (1, 1, 17)]
    for i, shp in enumerate(shapes):
        n = shp[-1]
        scores = torch.rand(*shp, generator=g)
        out[f"scores{i}"] = scores
        for how in ("mean", "max"):
            for prot_kind in ("count", "mask"):
                budget = max(1, n // 4)
                if prot_kind == "count":
                    prot = min(4, n)
                else:
                    prot = torch.rand(n, generator=g) < 0.1
                keep = keep_mask_from_scores(scores, n, budget, prot, how)
                key = f"k{len(names)}_"
                names.append([list(shp), how, prot_kind, budget, i])
                out.update({key + "keep": keep,
                            key + "prot": prot if isinstance(prot, torch.Tensor) else np.int64(prot)})
    save("keep_masks.npz", meta={"cases": names}, **out)


# --------------------------------------------------------------------------- LRFU / nucleus
def gen_lrfu():
    g = torch.Generator().manual_seed(13)
    out = {}
    tp = []
    for i, n in enumerate([1, 5, 64, 1000, 4096]):
        s = torch.rand(n, generator=g) ** 4
        if n > 4:
            s[torch.randperm(n, generator=g)[: n // 5]] = 0.0
        for p in (0.5, 0.9, 0.99):
            tp.append([n, p])
            key = f"t{len(tp) - 1}_"
            out[key + "s"] = s
            out[key + "mask"] = top_p_mask(s, p)
    # a multi-round ActionLRFU trace: observe a few action tokens, update, select, apply_keep
    rounds = []
    pol = ActionLRFU(EvictionConfig(decay=0.9, top_p=0.9))
    pol.reset(3)
    length = 50
    for rnd in range(4):
        pol.begin_action()
        obs = []
        for _ in range(3):
            sc = [torch.rand(length, generator=g) ** 3 for _ in range(3)]
            pol.observe(sc, True)
            obs.append(torch.stack(sc))
        keep = pol.select(length, protected=2, budget=30)
        key = f"r{rnd}_"
        out[key + "obs"] = torch.stack(obs)
        out[key + "length"] = np.int64(length)
        out[key + "ks"] = pol.ks.clone()
        out[key + "keep"] = keep if keep is not None else torch.zeros(0, dtype=torch.long)
        if keep is not None:
            pol.apply_keep(keep)
            out[key + "ks_after"] = pol.ks.clone()
            length = keep.shape[1]
        length += 20
        rounds.append(rnd)
    attn = torch.rand(8, 33, generator=g)
    out["rh_attn"] = attn
    out["rh_mean"] = reduce_heads(attn, 2, "mean")
    out["rh_max"] = reduce_heads(attn, 2, "max")
    save("lrfu.npz", meta={"top_p": tp, "rounds": len(rounds)}, **out)


# --------------------------------------------------------------------------- evict
def gen_evict():
    out = {}
    # multi-round evict with appends, pinned tokens carried across rounds
    case = cases.build_sessions(500, 2, 4, 2, 16, 16, [90, 45], [1, 1], extra_blocks=20)
    cache = ref_cache(case)
    g = torch.Generator().manual_seed(17)
    out["kv0_sha"] = np.array(cases.digest(cache.kv))
    out["free0"] = np.asarray(cache.free, np.int64)
    for r in range(2):
        out[f"table0_{r}"] = np.asarray(cache.tables[r], np.int64)
    step = 0
    for rnd in range(3):
        for r in range(2):
            n = cache.seq_used[r]
            scores = torch.rand(2, 2, n, generator=g)
            budget = [30, 12][r]
            perm = cache.evict(r, scores, budget, protected=5)
            key = f"s{step}_"
            out[key + "scores"] = scores
            out[key + "budget"] = np.int64(budget)
            out[key + "perm"] = perm
            out[key + "req"] = np.int64(r)
            out[key + "kv_sha"] = np.array(cases.digest(cache.kv))
            out[key + "free"] = np.asarray(cache.free, np.int64)
            out[key + "table"] = np.asarray(cache.tables[r], np.int64)
            out[key + "pinned"] = cache.pinned[r].clone()
            step += 1
            newk = torch.randn(2, 7 + r, 2, 16, generator=g)
            newv = torch.randn(2, 7 + r, 2, 16, generator=g)
            cache.append(r, newk, newv)
            out[key + "newk"] = newk
            out[key + "newv"] = newv
    save("evict.npz", meta={"steps": step}, **out)


# --------------------------------------------------------------------------- full pipelines
def run_pipeline(case, protected, budgets, decay, top_p, kv_digest_only):
    cache = ref_cache(case)
    kv0 = cache.kv.clone()
    res = {"kv_sha256_in": cases.digest(case.kv)}
    pols = []
    for r, (n, a) in enumerate(zip(case.seq_lens, case.act_lens)):
        pol = ActionLRFU(EvictionConfig(decay=decay, top_p=top_p))
        pol.reset(case.n_layers)
        pols.append(pol)
        bt = cache.block_table([r])
        width = bt.shape[1] * case.bs
        lse = torch.zeros(case.n_layers, a, case.hq)
        heads = torch.zeros(case.n_layers, case.hkv, n)
        for l in range(case.n_layers):
            o = torch.zeros(1, case.hkv, width)
            ns = torch.zeros(1, dtype=torch.int32)
            for j in range(a):
                seq = torch.tensor([n - a + j + 1], dtype=torch.int32)
                qj = case.q[r][l, j][None]
                _, lj = ref_lse.paged_decode_attention_ref(qj, cache.kv[l], bt, seq)
                lse[l, j] = lj[0]
                ref_lse.action_scores(qj, cache.kv[l], bt, seq, lj, o, ns)
            heads[l] = o[0, :, :n]
        act = heads.mean(1)                                   # reduce_heads "mean" per layer
        pol.act = act.clone()
        pol.n_act = a
        pol.update_scores(n, protected)
        ks = pol.ks.clone()
        keep = keep_mask_from_scores(ks, n, budgets[r], protected)
        table_before = list(cache.tables[r])
        plan = ref_compaction.plan_compaction(keep, n, torch.tensor(table_before), case.bs)
        perm = cache.evict(r, ks, budgets[r], protected)
        pol.apply_keep(perm.expand(case.n_layers, -1).contiguous())
        res.update({f"lse_{r}": lse, f"heads_{r}": heads, f"act_{r}": act, f"ks_{r}": ks,
                    f"keep_{r}": keep, f"perm_{r}": perm, f"src_{r}": plan.src_slots,
                    f"dst_{r}": plan.dst_slots, f"ks_after_{r}": pol.ks.clone(),
                    f"table_{r}": np.asarray(cache.tables[r], np.int64),
                    f"seq_{r}": np.int64(cache.seq_used[r]),
                    f"pinned_{r}": cache.pinned[r].clone()})
    res["free"] = np.asarray(cache.free, np.int64)
    res["kv_sha256_out"] = cases.digest(cache.kv)
    if not kv_digest_only:
        res["kv0"] = kv0
        res["kv1"] = cache.kv
    return res


def gen_pipelines():
    c1 = cases.build_sessions(**cases.CONFIG1)
    r1 = run_pipeline(c1, cases.CONFIG1_PROTECTED, [cases.CONFIG1_BUDGET], cases.CONFIG1_DECAY,
                      cases.CONFIG1_TOP_P, kv_digest_only=True)
    meta = {"kv_sha256_in": r1.pop("kv_sha256_in"), "kv_sha256_out": r1.pop("kv_sha256_out")}
    save("config1.npz", meta=meta, **r1)
    cb = cases.build_sessions(**cases.PIPE_BF16)
    rb = run_pipeline(cb, cases.PIPE_BF16_PROTECTED, cases.PIPE_BF16_BUDGETS, cases.PIPE_BF16_DECAY,
                      cases.PIPE_BF16_TOP_P, kv_digest_only=True)
    meta = {"kv_sha256_in": rb.pop("kv_sha256_in"), "kv_sha256_out": rb.pop("kv_sha256_out")}
    save("pipe_bf16.npz", meta=meta, **rb)



# --------------------------------------------------------------------------- adaptive budget
BUDGET_CONFIGS = [
    dict(),
    dict(init_budget=512, scale_up=1.75, upper=1000, window=4, stride=2),
    dict(init_budget=1000, window=16, stride=4, bottom_pct=50.0, bidirectional=True, shrink_patience=2,
         scale_down=2.0, lower=300),
    dict(init_budget=700, window=8, stride=3, bottom_pct=25.0, bidirectional=True, shrink_patience=1,
         shrink_slope=0.001),
]


def budget_logit_rows():
    """Logit rows for token_confidence: Gaussian of several widths, peaked, flat, exact ties at the
    top-k boundary, a row shorter than k, bf16-representable values."""
    g = torch.Generator().manual_seed(11)
    rows = [torch.randn(1000, generator=g) * s for s in (0.5, 2.0, 8.0)]
    rows.append(torch.cat([torch.tensor([12.0]), torch.zeros(999)]))
    rows.append(torch.zeros(1000))
    tie = torch.randn(1000, generator=g)
    tie[:40] = 3.0                                   # 40 equal values across the top-20 boundary
    rows.append(tie)
    rows.append(torch.randn(10, generator=g))        # fewer values than k
    rows.append((torch.randn(5000, generator=g) * 4).to(torch.bfloat16).float())
    return rows


def budget_traces():
    """Confidence traces and the number of values appended before each next_budget call."""
    g = torch.Generator().manual_seed(12)
    walk = torch.cumsum(torch.randn(600, generator=g) * 0.3, 0) + 20
    down = torch.linspace(30, 10, 400) + torch.randn(400, generator=g) * 0.5
    up = torch.linspace(10, 30, 400) + torch.randn(400, generator=g) * 0.5
    flat = torch.full((300,), 7.25)
    steps = [walk.float(), down.float(), up.float(), flat.float(),
             torch.tensor([5.0, 4.0, 6.0]).float()]
    chunks = [[0, 3, 40, 100, 200, 257], [50, 50, 100, 200], [64, 64, 64, 64, 144], [10, 90, 200], [3, 0]]
    return steps, chunks


def gen_budget():
    from actkv.budget import ConfidenceBudget, token_confidence
    from actkv.config import BudgetConfig
    rows = budget_logit_rows()
    out = {}
    for i, r in enumerate(rows):
        out[f"logits_{i}"] = r.numpy().astype(np.float32)
        out[f"conf_{i}"] = np.array([token_confidence(r, k) for k in (20, 5)], np.float64)
    traces, chunks = budget_traces()
    for t, (tl, ch) in enumerate(zip(traces, chunks)):
        out[f"trace_{t}"] = tl.numpy().astype(np.float32)
        out[f"chunks_{t}"] = np.array(ch, np.int64)
        for c, cfg in enumerate(BUDGET_CONFIGS):
            b = ConfidenceBudget(BudgetConfig(**cfg))
            got, slopes, n = [], [], 0
            for k in ch:
                b.tl.extend(float(v) for v in tl[n:n + k].tolist())
                n += k
                got.append(b.next_budget())
                slopes.append(b.slopes[-1])
            out[f"budgets_{t}_{c}"] = np.array(got, np.int64)
            out[f"slopes_{t}_{c}"] = np.array(slopes, np.float64)
    save("budget.npz", meta={"configs": BUDGET_CONFIGS, "n_rows": len(rows), "n_traces": len(traces),
                             "source": "actkv/budget.py token_confidence, ConfidenceBudget"}, **out)



# --------------------------------------------------------------------------- StreamingLLM / SnapKV
POLICY_CASES = [dict(window=4, pool=7), dict(window=6, pool=1), dict(window=3, pool=4), dict(window=32, pool=7)]


def policy_script(seed):
    """Observed rows of a 3-layer decode: 10 rows growing from 40 to 49 tokens, select at 50, then
    (after apply_keep) 5 rows growing from 25 to 29 tokens, select at 30."""
    g = torch.Generator().manual_seed(seed)
    first = [[torch.rand(40 + i, generator=g) for _ in range(3)] for i in range(10)]
    second = [[torch.rand(25 + i, generator=g) for _ in range(3)] for i in range(5)]
    return first, second


def gen_policies():
    from actkv.eviction import SnapKV, StreamingLLM
    out = {}
    first, second = policy_script(21)
    for i, rows in enumerate(first + second):
        for layer, r in enumerate(rows):
            out[f"row_{i}_{layer}"] = r.numpy()
    for c, cfg in enumerate(POLICY_CASES):
        pol = SnapKV(**cfg)
        pol.reset(3)
        for rows in first:
            pol.observe(rows, True)
        k1 = pol.select(50, protected=4, budget=20)
        pol.apply_keep(k1)
        for rows in second:
            pol.observe(rows, True)
        k2 = pol.select(30, protected=4, budget=12)
        k3 = pol.select(30, protected=4, budget=30)          # within budget: None
        out[f"snap_{c}_k1"], out[f"snap_{c}_k2"] = k1.numpy(), k2.numpy()
        out[f"snap_{c}_none"] = np.array(k3 is None)
    st = StreamingLLM()
    st.reset(3)
    out["stream_k"] = st.select(50, protected=4, budget=20).numpy()
    out["stream_none"] = np.array(st.select(24, protected=4, budget=20) is None)
    save("policies.npz", meta={"cases": POLICY_CASES, "n_rows": len(first) + len(second), "n_layers": 3,
                               "source": "actkv/eviction.py SnapKV, StreamingLLM"}, **out)



# --------------------------------------------------------------------------- decode attention
DECODE_CASES = [
    dict(seed=51, n_layers=1, hq=8, hkv=2, d=128, bs=16, seq_lens=[300, 517, 40], act_lens=[1, 1, 1],
         dtype="bfloat16", extra_blocks=4),
    dict(seed=52, n_layers=1, hq=32, hkv=8, d=128, bs=16, seq_lens=[9000, 1], act_lens=[1, 1],
         dtype="float16", extra_blocks=2),
    dict(seed=53, n_layers=1, hq=4, hkv=4, d=64, bs=8, seq_lens=[77, 200], act_lens=[1, 1],
         dtype="float32", extra_blocks=2),
]


def gen_decode():
    """(out, lse) of the reference's paged_decode_attention_ref for one query per session."""
    out = {}
    for c, spec in enumerate(DECODE_CASES):
        case = cases.build_sessions(**spec)
        q = torch.cat([qq[0] for qq in case.q], 0)                 # [R, Hq, D]
        bt = torch.from_numpy(cases.block_table_array(case.tables))
        seq = torch.tensor(case.seq_lens, dtype=torch.int32)
        o, lse = ref_lse.paged_decode_attention_ref(q, case.kv[0], bt, seq)
        out[f"out_{c}"], out[f"lse_{c}"] = o.numpy(), lse.numpy()
        out[f"kv_sha_{c}"] = np.array(cases.digest(case.kv))
    save("decode.npz", meta={"cases": DECODE_CASES, "source": "actkv/kernels/lse_attn.py paged_decode_attention_ref"},
         **out)


if __name__ == "__main__":
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    gen_scores()
    gen_plans()
    gen_compact()
    gen_keep_masks()
    gen_lrfu()
    gen_evict()
    gen_pipelines()
    gen_budget()
    gen_policies()
    gen_decode()
