"""Sharded hot path on the GPU: the head-shard reassembly kernel, and every rank's part of a
sharded image computed on one device, gathered and reassembled, equal to the single-GPU path.

The all-gather between ranks is emulated here by concatenating the rank blocks in rank order
(exactly what ``all_gather_into_tensor`` produces); the NCCL path itself runs in
``test_gpu_multi.py`` when two GPUs are present.
"""

import ctypes

import numpy as np
import pytest
import torch

import bench
from heatkv_b200 import _native, sharding
from heatkv_b200.hotpath import HotPath, allocate_io

pytestmark = pytest.mark.gpu

DT = _native.DTYPE_CODES


def _gather(full, recv, world, rpr, n, hpr, batch, heads, row_map, head_map):
    lib = _native.load()
    st = lib.heatkv_gather_head_shards(
        _native.ptr(full), _native.ptr(recv), DT[full.dtype], world, rpr, n, hpr, batch, heads,
        128, _native.ptr(row_map), _native.ptr(head_map), _native.stream_handle(full.device))
    _native.check(st, "gather head shards")


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("world,rpr,hpr,n", [(2, 2, 8, 4096), (8, 1, 4, 576), (4, 1, 4, 1)])
def test_gather_head_shards_matches_indexing(dtype, world, rpr, hpr, n):
    """rank r holds rows of row group r // (H / hpr) and a permuted head group r % (H / hpr)."""
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(world * 100 + n)
    heads = 16
    hg = heads // hpr
    batch = (world // hg) * rpr
    perm = np.random.default_rng(n).permutation(heads)
    row_map = np.array([(r // hg) * rpr + i for r in range(world) for i in range(rpr)], np.int32)
    head_map = np.array([perm[(r % hg) * hpr + j] for r in range(world) for j in range(hpr)],
                        np.int32)
    recv = torch.randn(world, rpr, n, hpr * 128, device=dev, generator=g).to(dtype)
    full = torch.full((batch, n, heads * 128), float("nan"), device=dev, dtype=dtype)
    _gather(full, recv, world, rpr, n, hpr, batch, heads, torch.from_numpy(row_map).to(dev),
            torch.from_numpy(head_map).to(dev))
    torch.cuda.synchronize()
    ref = torch.empty_like(full)
    for r in range(world):
        for i in range(rpr):
            for j in range(hpr):
                h = int(head_map[r * hpr + j])
                ref[int(row_map[r * rpr + i]), :, h * 128:(h + 1) * 128] = \
                    recv[r, i, :, j * 128:(j + 1) * 128]
    assert torch.equal(full, ref)
    assert _native.device_status(dev) == 0


def test_gather_head_shards_flags_out_of_range_maps():
    dev = torch.device("cuda", 0)
    recv = torch.ones(2, 1, 8, 8 * 128, device=dev, dtype=torch.bfloat16)
    full = torch.zeros(2, 8, 16 * 128, device=dev, dtype=torch.bfloat16)
    rm = torch.tensor([0, 1], dtype=torch.int32, device=dev)
    hm = torch.tensor(list(range(8)) + [8, 9, 10, 11, 12, 13, 14, 99], dtype=torch.int32,
                      device=dev)
    _gather(full, recv, 2, 1, 8, 8, 2, 16, rm, hm)
    torch.cuda.synchronize()
    assert _native.device_status(dev) == _native.DEVICE_GATHER_OUT_OF_RANGE
    # every in-range chunk was written, the bad one skipped
    assert full[1, :, 15 * 128:].abs().sum().item() == 0
    assert full[1, :, 8 * 128:15 * 128].eq(1).all()
    assert full[0, :, :8 * 128].eq(1).all()


@pytest.mark.parametrize("world,split", [(2, "heads"), (4, "auto"), (8, "heads")])
def test_sharded_ranks_reassemble_the_single_gpu_outputs(world, split):
    dev = torch.device("cuda", 0)
    ctrl, L, H = bench.build_controller("2b", 0.10)
    layers = [0, 21]
    batch = 2
    # no key-range splits on either side: a split block sums in a different order
    full = HotPath(ctrl, L, H, batch, dev, layers=layers, plan_splits=1)
    inputs, outputs, _, _ = allocate_io(full, seed=5)
    HotPath.run(full.launches(inputs, outputs))
    costs = sharding.head_costs(ctrl, L, H)
    plan = sharding.plan_shards(costs, batch, world, split=split)
    assert plan.splits_heads
    ranks = [sharding.ShardedHotPath(ctrl, L, H, plan, r, dev, layers=layers, plan_splits=1)
             for r in range(world)]
    local_out = []
    for r, sh in enumerate(ranks):
        rows = plan.rows_of(r)
        li, lo = [], []
        for i, layer in enumerate(layers):
            hs = torch.tensor(plan.heads_of(r, layer), device=dev)
            li.append([tuple(x[rows[0]:rows[-1] + 1].index_select(1, hs).contiguous()
                             for x in inputs[i][t]) for t in range(full.num_scales)])
            lo.append([torch.empty(plan.rows_per_rank, full.tokens[t],
                                   plan.heads_per_rank * 128, device=dev, dtype=torch.bfloat16)
                       for t in range(full.num_scales)])
        HotPath.run(sh.local.launches(li, lo))
        local_out.append((li, lo))
    torch.cuda.synchronize()
    for i, layer in enumerate(layers):
        hm = ranks[0].head_maps[layer]
        for t in range(full.num_scales):
            n = full.tokens[t]
            recv = torch.cat([local_out[r][1][i][t].unsqueeze(0) for r in range(world)])
            got = torch.full_like(outputs[i][t], float("nan"))
            _gather(got, recv, world, plan.rows_per_rank, n, plan.heads_per_rank, batch, H,
                    ranks[0].row_map, hm)
            torch.cuda.synchronize()
            # the same (row, head) units with the same keys in the same order: identical bits
            assert torch.equal(got, outputs[i][t]), (layer, t)
    assert _native.device_status(dev) == 0


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("mapped", [False, True])
def test_scatter_attention_places_rows_in_every_destination(mapped, dtype):
    """heatkv_segmented_attention_scatter: the heads of one call split over two emulated ranks,
    each storing its rows into two full outputs (both on this GPU; one 32-byte aligned, one only
    16-byte aligned), equals the unsharded call of the kernel the scatter runs (the 64-key one,
    unsplit), bit for bit. ``mapped``: heatkv_segmented_attention_scatter_mapped with a random
    assignment of the items to 37 CTAs (empty slots included) - a schedule only, same bits."""
    dev = torch.device("cuda", 0)
    lib = _native.load()
    B, H, L, cap, S = 2, 16, 600, 5000, 8
    rng = np.random.default_rng(17)
    gen = torch.Generator().manual_seed(17)
    q, k, v = (torch.randn(B, H, L, 128, generator=gen).to(dtype).to(dev) for _ in range(3))
    pk, pv = (torch.randn(B, cap, 128, generator=gen).to(dtype).to(dev) for _ in range(2))
    st = np.zeros((H, S), np.int32)
    en = np.zeros((H, S), np.int32)
    ct = rng.integers(0, S + 1, size=H).astype(np.int32)
    for h in range(H):
        for i in range(ct[h]):
            n = int(rng.choice([1, 4, 64, 130, 576]))
            s0 = int(rng.integers(0, cap - n + 1))
            st[h, i], en[h, i] = s0, s0 + n
    scale = ctypes.c_float(128 ** -0.5)
    ref = torch.empty(B, L, H * 128, dtype=dtype, device=dev)
    meta = [torch.from_numpy(x).to(dev) for x in (st, en, ct)]
    _native.check(lib.heatkv_segmented_attention(
        _native.ptr(q), _native.ptr(pk), _native.ptr(pv), *[_native.ptr(m) for m in meta],
        _native.ptr(k), _native.ptr(v), _native.ptr(ref), DT[q.dtype], DT[k.dtype], DT[v.dtype],
        B, H, L, cap, 128, S, scale, 0, _native.ATTN_TCGEN05_CS64,
        _native.stream_handle(dev)), "reference call")
    # the second destination starts 16 bytes into its buffer: the epilogue's 16-byte stores
    spare = torch.full((ref.numel() + 8,), float("nan"), dtype=ref.dtype, device=dev)
    dests = [torch.full_like(ref, float("nan")), spare[8:].view(ref.shape)]
    assert dests[1].data_ptr() % 32 == 16
    ptrs = torch.tensor([d.data_ptr() for d in dests], dtype=torch.int64, device=dev)
    rows = torch.arange(B, dtype=torch.int32, device=dev)
    groups = [sorted(rng.permutation(H)[:H // 2].tolist())]
    groups.append(sorted(set(range(H)) - set(groups[0])))
    for hs in groups:
        idx = torch.tensor(hs, device=dev)
        qs, ks, vs = (x.index_select(1, idx).contiguous() for x in (q, k, v))
        ms = [m.index_select(0, idx).contiguous() for m in meta]
        heads = torch.tensor(hs, dtype=torch.int32, device=dev)
        args = (_native.ptr(qs), _native.ptr(pk), _native.ptr(pv), *[_native.ptr(m) for m in ms],
                _native.ptr(ks), _native.ptr(vs), _native.ptr(ptrs), 2, _native.ptr(rows),
                _native.ptr(heads), B, H, DT[q.dtype], DT[k.dtype], DT[v.dtype], B, len(hs), L,
                cap, 128, S, scale, None)
        if mapped:
            items = B * len(hs) * ((L + 127) // 128)
            grid = 37
            slots = np.full(((items + 9 + grid - 1) // grid) * grid, -1, np.int32)
            slots[rng.permutation(slots.size)[:items]] = rng.permutation(items)
            imap = torch.from_numpy(slots).to(dev)
            _native.check(lib.heatkv_segmented_attention_scatter_mapped(
                *args, _native.ptr(imap), imap.numel(), grid, _native.stream_handle(dev)),
                "mapped scatter call")
            torch.cuda.synchronize()
        else:
            _native.check(lib.heatkv_segmented_attention_scatter(
                *args, _native.stream_handle(dev)), "scatter call")
    torch.cuda.synchronize()
    for d in dests:
        assert torch.equal(d, ref)
    assert _native.device_status(dev) == 0


def test_scatter_skips_and_flags_rows_mapped_outside_the_full_output():
    """A local row or head whose mapped place lies outside the full output is not stored (the
    epilogue checks the maps before every store) and raises HEATKV_DEVICE_GATHER_OUT_OF_RANGE;
    the other rows land where their maps say."""
    dev = torch.device("cuda", 0)
    lib = _native.load()
    B, H, L = 2, 4, 130
    gen = torch.Generator().manual_seed(5)
    q, k, v = (torch.randn(B, H, L, 128, generator=gen).bfloat16().to(dev) for _ in range(3))
    st = torch.zeros(H, 1, dtype=torch.int32, device=dev)
    ct = torch.zeros(H, dtype=torch.int32, device=dev)     # current keys only
    scale = ctypes.c_float(128 ** -0.5)
    ref = torch.empty(B, L, H * 128, dtype=torch.bfloat16, device=dev)
    _native.check(lib.heatkv_segmented_attention(
        _native.ptr(q), None, None, _native.ptr(st), _native.ptr(st), _native.ptr(ct),
        _native.ptr(k), _native.ptr(v), _native.ptr(ref), DT[q.dtype], DT[k.dtype], DT[v.dtype],
        B, H, L, 0, 128, 1, scale, 0, _native.ATTN_TCGEN05_CS64,
        _native.stream_handle(dev)), "reference call")
    out = torch.full_like(ref, float("nan"))
    ptrs = torch.tensor([out.data_ptr()], dtype=torch.int64, device=dev)
    rows = torch.tensor([1, 7], dtype=torch.int32, device=dev)       # row 1 -> 7: outside
    heads = torch.tensor([3, 2, -1, 0], dtype=torch.int32, device=dev)  # head 2 -> -1: outside
    _native.check(lib.heatkv_segmented_attention_scatter(
        _native.ptr(q), None, None, _native.ptr(st), _native.ptr(st), _native.ptr(ct),
        _native.ptr(k), _native.ptr(v), _native.ptr(ptrs), 1, _native.ptr(rows), _native.ptr(heads),
        B, H, DT[q.dtype], DT[k.dtype], DT[v.dtype], B, H, L, 0, 128, 1, scale, None,
        _native.stream_handle(dev)), "scatter call")
    torch.cuda.synchronize()
    ref4 = ref.view(B, L, H, 128)
    out4 = out.view(B, L, H, 128)
    for h, g in ((0, 3), (1, 2), (3, 0)):
        assert torch.equal(out4[1, :, g], ref4[0, :, h])
    assert torch.isnan(out4[0]).all()        # nothing maps to row 0
    assert torch.isnan(out4[1, :, 1]).all()  # the head mapped outside
    assert _native.device_status(dev) == _native.DEVICE_GATHER_OUT_OF_RANGE


def test_scatter_of_dense_launches_uses_prefix_only_segments():
    """The hot path's dense-prefix launches walk one segment per head that already ends with the
    current scale (HEATKV_ATTN_CURRENT_IN_SEGMENTS). The scatter entry point of the peer-to-peer
    exchange takes no kernel selector, so the exchange re-issues those launches with their
    prefix-only segments (Launch.unflagged_meta). Re-issued that way into one full output on this
    GPU, every dense target of a layer matches the hot path's own output (bf16 tolerance: the
    re-issued launch splits its keys into tiles at other places) and, bit for bit, the hot path
    built without dense appends first (the reference the 2-GPU peer-to-peer test compares
    with)."""
    dev = torch.device("cuda", 0)
    lib = _native.load()
    ctrl, L, H = bench.build_controller("2b", 0.10)
    hot = HotPath(ctrl, L, H, 2, dev, layers=[21], plan_splits=1)
    inputs, outputs, _, _ = allocate_io(hot, seed=4)
    launches = hot.launches(inputs, outputs)
    HotPath.run(launches)
    plain = HotPath(ctrl, L, H, 2, dev, layers=[21], plan_splits=1, dense_append_first=False)
    _, plain_out, _, _ = allocate_io(plain, seed=4, fill=False)
    HotPath.run(plain.launches(inputs, plain_out))
    torch.cuda.synchronize()
    rows = torch.arange(2, dtype=torch.int32, device=dev)
    heads = torch.arange(H, dtype=torch.int32, device=dev)
    checked = 0
    for launch in launches:
        # dense targets only: their dense-cache rows stay as they were; later appends reuse the
        # slots of fused targets, so those cannot be re-run after the step
        if launch.kind != "attention" or launch.target >= hot.plans[0].first_target:
            continue
        a = launch.args
        meta = launch.unflagged_meta or (a[3], a[4], a[5])
        if launch.target in hot.plans[0].dense_append:
            assert launch.unflagged_meta is not None
        ref = outputs[0][launch.target]
        out = torch.full_like(ref, float("nan"))
        ptrs = torch.tensor([out.data_ptr()], dtype=torch.int64, device=dev)
        _native.check(lib.heatkv_segmented_attention_scatter(
            a[0], a[1], a[2], meta[0], meta[1], meta[2], a[6], a[7], _native.ptr(ptrs), 1,
            _native.ptr(rows), _native.ptr(heads), 2, H, a[9], a[10], a[11], a[12], a[13], a[14],
            a[15], a[16], a[17], a[18], a[20], _native.stream_handle(dev)), "scatter")
        torch.cuda.synchronize()
        err = (out.float() - ref.float()).abs().max().item()
        assert err <= 2e-2 and err / ref.float().abs().max().item() <= 1e-2, (launch.target, err)
        assert torch.equal(out, plain_out[0][launch.target]), launch.target
        checked += 1
    assert checked >= 7
    assert _native.device_status(dev) == 0
