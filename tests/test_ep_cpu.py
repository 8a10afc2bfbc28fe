"""Expert-parallel host logic on the CPU: row and expert ownership, the
exchange arithmetic (restated here in numpy: each rank's per-expert segments,
the receive layout of every rank's experts, and where the down GEMM stores
each received row's output — home, at the row's position in its source's
permuted layout) checked against the single-GPU permutation, and the same
arithmetic run by two gloo ranks that exchange their counts as the GPUs do."""
import os
import socket

import numpy as np
import pytest

import ep


def test_rows_of_partitions_every_row_once():
    for total in (0, 1, 7, 32768, 32769):
        for world in (1, 2, 3, 8):
            spans = [ep.rows_of(total, world, r) for r in range(world)]
            assert sum(c for _, c in spans) == total
            pos = 0
            for s, c in spans:
                assert s == pos
                pos += c
            assert max(c for _, c in spans) - min(c for _, c in spans) <= 1


@pytest.mark.parametrize("strided", [False, True])
def test_expert_ownership(strided):
    for E, W in ((64, 1), (64, 2), (64, 8), (16, 4), (128, 8)):
        owned = [ep.local_experts(r, E, W, strided) for r in range(W)]
        assert sorted(e for o in owned for e in o) == list(range(E))
        for r, o in enumerate(owned):
            assert o == sorted(o) and len(o) == E // W
            assert all(ep.expert_owner(e, E, W, strided) == r for e in o)


# ---- the exchange arithmetic -------------------------------------------------

def permute(ids, E):
    """The single-GPU stable permutation: (seg_count, seg_start, pos_of)."""
    flat = ids.ravel()
    seg_count = np.bincount(flat, minlength=E)
    seg_start = np.concatenate([[0], np.cumsum(seg_count)[:-1]])
    order = np.argsort(flat, kind="stable")
    pos = np.empty(flat.size, np.int64)
    pos[order] = np.arange(flat.size)
    return seg_count, seg_start, pos.reshape(ids.shape)


def receive_layout(cnt_all, W, E, strided):
    """rstart[d][i]: first row of rank d's local expert i in d's receive
    buffer; tot[d][i] its row count (the prepare kernel's tables)."""
    L = E // W
    tot = np.zeros((W, L), np.int64)
    for d in range(W):
        for i, e in enumerate(ep.local_experts(d, E, W, strided)):
            tot[d, i] = cnt_all[:, e].sum()
    rstart = np.concatenate([np.zeros((W, 1), np.int64), np.cumsum(tot, axis=1)[:, :-1]], axis=1)
    return tot, rstart


def segments(d, cnt_all, seg_start_all, rstart, W, E, strided):
    """Rank d's (slot, source) segments as the prepare kernel lays them out:
    (first receive row, first row in the source's xperm, source), slot-major."""
    segs = []
    for i, e in enumerate(ep.local_experts(d, E, W, strided)):
        for s in range(W):
            segs.append((int(rstart[d, i] + cnt_all[:s, e].sum()), int(seg_start_all[s, e]), s))
    return segs


def home_of(segs, r):
    """The scatter of the down GEMM's epilogue: receive row r goes to row
    seg_src + r - seg_dst of the last segment starting at or before r."""
    dst, src, s = [g for g in segs if g[0] <= r][-1]
    return s, src + r - dst


def simulate(ids_per_rank, W, E, strided):
    """Per-rank permutations, the pulls into every owner's receive rows, and
    where each received row's output goes home. Returns, per owner, the
    (source rank, row) of each received row and the (source rank, position)
    its output is stored at."""
    perms = [permute(ids, E) for ids in ids_per_rank]
    cnt_all = np.stack([p[0] for p in perms])
    seg_start_all = np.stack([p[1] for p in perms])
    tot, rstart = receive_layout(cnt_all, W, E, strided)
    recv, home = [], []
    for d in range(W):
        rows = []
        for i, e in enumerate(ep.local_experts(d, E, W, strided)):
            for s in range(W):
                seg_count, seg_start, pos = perms[s]
                # rows of s's xperm segment e, in segment order = token order
                toks = np.argsort(ids_per_rank[s].ravel(), kind="stable")[seg_start[e]:seg_start[e] + seg_count[e]]
                rows += [(s, int(t) // ids_per_rank[s].shape[1]) for t in toks]
        assert len(rows) == tot[d].sum()
        recv.append(rows)
        segs = segments(d, cnt_all, seg_start_all, rstart, W, E, strided)
        home.append([home_of(segs, r) for r in range(len(rows))])
    return recv, home, perms


def check_homes(ids_per_rank, recv, home, perms, W, E, strided):
    """Every selection's output lands exactly once, at its own position of its
    source's permuted layout (where the single-GPU combine reads it), and the
    row stored there is the one that was pulled."""
    landed = [dict() for _ in range(W)]
    for d in range(W):
        for r, ((s, t), (hs, p)) in enumerate(zip(recv[d], home[d])):
            assert hs == s
            assert p not in landed[s]
            landed[s][p] = t
    for s in range(W):
        n = len(ids_per_rank[s])
        assert len(landed[s]) == n * ids_per_rank[s].shape[1]
        pos = perms[s][2]
        for t in range(n):
            for j in range(ids_per_rank[s].shape[1]):
                assert landed[s][int(pos[t, j])] == t


def first_positions(ids, pos, rank, W, E, strided):
    """ep_first_kernel: per xperm position of `rank`, the position of the same
    row's selection with the lowest expert id among those one owner takes."""
    first = np.full(ids.size, -1, np.int64)
    for t in range(ids.shape[0]):
        owners = [ep.expert_owner(int(e), E, W, strided) for e in ids[t]]
        for j, e in enumerate(ids[t]):
            same = [i for i in range(ids.shape[1]) if owners[i] == owners[j]]
            best = min(same, key=lambda i: ids[t, i])
            first[pos[t, j]] = pos[t, best]
    return first


def pull_plan(d, recv_rows, segs, seg_start_all, firsts, W, E, strided):
    """ep_pull_kernel's choice per receive row of rank d: -1 = pulled over
    NVLink, else the earlier receive row it is copied from (ep_dup_kernel)."""
    plan = []
    for r in range(len(recv_rows)):
        dst, src, s = [g for g in segs if g[0] <= r][-1]
        p = src + r - dst
        fp = int(firsts[s][p])
        frm = -1
        if 0 <= fp < p:
            a = max(e for e in range(E) if seg_start_all[s, e] <= fp)
            if ep.expert_owner(a, E, W, strided) == d:
                i = ep.local_experts(d, E, W, strided).index(a)
                q = i * W + s
                r0 = segs[q][0] + fp - segs[q][1]
                if 0 <= r0 < r:
                    frm = r0
        plan.append(frm)
    return plan


@pytest.mark.parametrize("W,strided", [(2, False), (4, True), (8, False)])
def test_each_row_crosses_once_per_owner(W, strided):
    """The deduplicated pull: every (source row, owner) pair is pulled exactly
    once, and every other receive row of the same source row copies a pulled
    row holding the same source row — xrecv ends up as the full pull."""
    rng = np.random.default_rng(7 + W)
    E, K = 32, 6
    rows = rng.integers(20, 60, size=W)
    ids_per_rank = [np.stack([rng.choice(E, K, replace=False) for _ in range(n)]).astype(np.int64) for n in rows]
    recv, _, perms = simulate(ids_per_rank, W, E, strided)
    cnt_all = np.stack([p[0] for p in perms])
    seg_start_all = np.stack([p[1] for p in perms])
    _, rstart = receive_layout(cnt_all, W, E, strided)
    firsts = [first_positions(ids_per_rank[s], perms[s][2], s, W, E, strided) for s in range(W)]
    pulled_total = sel_total = 0
    for d in range(W):
        segs = segments(d, cnt_all, seg_start_all, rstart, W, E, strided)
        plan = pull_plan(d, recv[d], segs, seg_start_all, firsts, W, E, strided)
        pulled = [recv[d][r] for r in range(len(plan)) if plan[r] < 0]
        assert len(pulled) == len(set(pulled)) == len(set(recv[d]))
        for r, frm in enumerate(plan):
            if frm >= 0:
                assert plan[frm] < 0 and recv[d][frm] == recv[d][r]
        pulled_total += sum(1 for (s, _), f in zip(recv[d], plan) if f < 0 and s != d)
        sel_total += sum(1 for s, _ in recv[d] if s != d)
    assert pulled_total < sel_total  # rows with several experts on one owner cross once


@pytest.mark.parametrize("W,strided", [(2, False), (4, True), (8, False)])
def test_pull_byte_count_matches_the_pull_plan(W, strided):
    """ep.rows_pulled_from (the bench's NVLink byte count) equals the rows the
    deduplicated pull plan moves from each source to each owner."""
    rng = np.random.default_rng(11 + W)
    E, K = 32, 6
    rows = rng.integers(10, 40, size=W)
    ids_per_rank = [np.stack([rng.choice(E, K, replace=False) for _ in range(n)]).astype(np.int64) for n in rows]
    recv, _, perms = simulate(ids_per_rank, W, E, strided)
    cnt_all = np.stack([p[0] for p in perms])
    seg_start_all = np.stack([p[1] for p in perms])
    _, rstart = receive_layout(cnt_all, W, E, strided)
    firsts = [first_positions(ids_per_rank[s], perms[s][2], s, W, E, strided) for s in range(W)]
    owner = ep.owner_table(E, W, strided)
    for d in range(W):
        segs = segments(d, cnt_all, seg_start_all, rstart, W, E, strided)
        plan = pull_plan(d, recv[d], segs, seg_start_all, firsts, W, E, strided)
        for s in range(W):
            moved = sum(1 for (src, _), f in zip(recv[d], plan) if src == s and f < 0) if s != d else 0
            assert moved == ep.rows_pulled_from(ids_per_rank[s], owner, W, s)[d]


@pytest.mark.parametrize("W,strided", [(2, False), (4, True), (8, False), (8, True)])
def test_exchange_arithmetic_reproduces_single_gpu_order(W, strided):
    rng = np.random.default_rng(W)
    E, K = 32, 4
    rows = rng.integers(0, 50, size=W)
    rows[0] = 0  # an empty rank still takes part
    p = 1.0 / np.arange(1, E + 1) ** 1.2
    ids_per_rank = [np.stack([rng.choice(E, K, replace=False, p=p / p.sum()) for _ in range(n)]).astype(np.int64)
                    if n else np.zeros((0, K), np.int64) for n in rows]
    recv, home, perms = simulate(ids_per_rank, W, E, strided)
    offsets = np.concatenate([[0], np.cumsum(rows)])
    glob_ids = np.concatenate(ids_per_rank)
    for d in range(W):
        # Each expert's received rows are its selections in global row order,
        # exactly the rows a single GPU puts in that expert's segment.
        got = [offsets[s] + t for s, t in recv[d]]
        want = []
        for e in ep.local_experts(d, E, W, strided):
            want += [t for t in range(len(glob_ids)) if e in glob_ids[t]]
        assert got == want
    check_homes(ids_per_rank, recv, home, perms, W, E, strided)


# ---- two gloo ranks ----------------------------------------------------------

def _free_port():
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        return sk.getsockname()[1]


def _gloo_rank(rank, world, port, E, K, strided, result_q):
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        rng = np.random.default_rng(100 + rank)
        n = [37, 0, 12][rank % 3]
        ids = np.stack([rng.choice(E, K, replace=False) for _ in range(n)]).astype(np.int64) if n else \
            np.zeros((0, K), np.int64)
        seg_count, seg_start, pos = permute(ids, E)
        # the counts exchange the prepare kernel does with peer loads
        allc = [torch.zeros(E, dtype=torch.int64) for _ in range(world)]
        dist.all_gather(allc, torch.from_numpy(seg_count))
        alls = [torch.zeros(E, dtype=torch.int64) for _ in range(world)]
        dist.all_gather(alls, torch.from_numpy(seg_start))
        cnt_all = torch.stack(allc).numpy()
        seg_start_all = torch.stack(alls).numpy()
        _, rstart = receive_layout(cnt_all, world, E, strided)
        # this rank's own (slot, source) segments, from the exchanged counts only
        mine = segments(rank, cnt_all, seg_start_all, rstart, world, E, strided)
        # handles travel as opaque bytes, in rank order
        handles = ep.exchange_handles(bytes([rank]) * 256)
        assert [h[0] for h in handles] == list(range(world))
        obj = [None] * world
        dist.all_gather_object(obj, (ids, mine))
        if rank == 0:
            ids_all = [o[0] for o in obj]
            recv, home, perms = simulate(ids_all, world, E, strided)
            ok = True
            for d in range(world):
                segs_d = obj[d][1]
                ok &= [home_of(segs_d, r) for r in range(len(recv[d]))] == home[d]
            check_homes(ids_all, recv, home, perms, world, E, strided)
            result_q.put(bool(ok))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("strided", [False, True])
def test_two_gloo_ranks_agree_with_one_process(strided):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gloo_rank, args=(r, 2, port, 16, 3, strided, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
    assert all(p.exitcode == 0 for p in procs)
    assert q.get(timeout=5) is True


# ---- load-balanced placement ----------------------------------------------

# Rows per expert of the config-3 prefill layer (32768 rows, top-6, the
# Zipf(1.2)-biased router), as the bench measured them on B200.
C3_HISTOGRAM = [26872, 21042, 16749, 13694, 11519, 10011, 8258, 7256, 6636, 5722, 4861, 4539, 4174, 3601, 3388, 3118,
                2828, 2627, 2452, 2226, 2118, 1845, 1820, 1751, 1707, 1393, 1321, 1474, 1294, 1281, 1074, 1103, 808,
                869, 959, 782, 836, 733, 641, 698, 717, 606, 643, 638, 557, 534, 507, 495, 557, 487, 422, 445, 408,
                455, 348, 357, 378, 315, 310, 325, 270, 233, 270, 251]


def _by_source(hist, W):
    return [[h // W + (1 if s < h % W else 0) for h in hist] for s in range(W)]


@pytest.mark.parametrize("W", [2, 4, 8])
def test_balanced_owner_table_evens_out_the_received_rows(W):
    E = len(C3_HISTOGRAM)
    cbs = _by_source(C3_HISTOGRAM, W)
    owner = ep.balanced_owner_table(cbs, W)
    assert len(owner) == E * W and all(0 <= d < W for d in owner)
    got = ep.rows_received(owner, cbs, E, W)
    assert sum(got) == sum(C3_HISTOGRAM)
    assert max(got) / (sum(got) / W) <= 1.05
    # the built-in maps are far off on this histogram
    assert max(ep.rows_received(ep.owner_table(E, W, True), cbs, E, W)) / (sum(got) / W) > 1.07
    for d in range(W):
        assert len(ep.slots_of(owner, E, W, d)) >= 1
    for e in range(E):
        reps = sorted({owner[e * W + s] for s in range(W)})
        assert W % len(reps) == 0  # replicas split the sources evenly
        for s in range(W):  # replica j takes the sources s % r == j
            assert owner[e * W + s] == owner[e * W + s % len(reps)]
    assert ep.balanced_owner_table(cbs, W) == owner  # deterministic: every rank computes the same table


def test_owner_table_matches_the_built_in_maps():
    for E, W in ((64, 8), (16, 4)):
        for strided in (False, True):
            owner = ep.owner_table(E, W, strided)
            for d in range(W):
                assert ep.slots_of(owner, E, W, d) == ep.local_experts(d, E, W, strided)


def test_balanced_table_with_more_ranks_than_hot_experts():
    cbs = _by_source([1000, 1, 1], 4)
    owner = ep.balanced_owner_table(cbs, 4)
    assert all(len(ep.slots_of(owner, 3, 4, d)) >= 1 for d in range(4))
