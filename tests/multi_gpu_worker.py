"""One rank of the multi-GPU parity check (launched by test_gpu_multi.py under torchrun).

Every rank builds the same seeded global inputs of two 2B layers, keeps its (row, head) units,
runs its part of the sharded hot path - attention, compaction, NCCL all-gather and reassembly -
eagerly and then as a CUDA graph replay, and checks that the full outputs it received equal the
single-GPU engine's outputs bit for bit. Rank 0 also checks the gathered outputs of one layer at
every scale against attention over exactly the tokens the keep-mask retains (plain PyTorch fp32,
``_keepmask.keep_mask_attention``) at the bf16 tolerance, so the exchange is pinned to the
keep-mask semantics and not only to the engine it mirrors. Exit status 0 = parity.
"""

import datetime
import os
import sys

import torch
import torch.distributed as dist

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
sys.path.insert(0, REPO)
sys.path.insert(0, HERE)

import bench  # noqa: E402
from heatkv_b200 import _native, sharding  # noqa: E402
from heatkv_b200.hotpath import HotPath, allocate_io  # noqa: E402
from _keepmask import keep_mask_attention  # noqa: E402

BF16_ATOL, BF16_REL = 2e-2, 1e-2


def main() -> int:
    split = sys.argv[1] if len(sys.argv) > 1 else "heads"
    exchange = sys.argv[2] if len(sys.argv) > 2 else "nccl"
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    ok = True
    try:
        ctrl, L, H = bench.build_controller("2b", 0.10)
        layers, batch = [0, 21], 2
        # no key-range splits on either side: a split block sums in a different order
        # the peer-to-peer exchange scatters from the 64-key kernel unsplit, over prefix-only
        # dense segments followed by the current tiles: compare bits with exactly that
        p2p = exchange == "p2p"
        full = HotPath(ctrl, L, H, batch, dev, layers=layers, plan_splits=1,
                       dense_append_first=not p2p)
        inputs, ref_out, _, _ = allocate_io(full, seed=11)       # identical on every rank
        HotPath.run(full.launches(inputs, ref_out, kernel=_native.ATTN_AUTO))
        plan = sharding.plan_shards(sharding.head_costs(ctrl, L, H), batch, world, split=split)
        sh = sharding.ShardedHotPath(ctrl, L, H, plan, rank, dev, gather=True, layers=layers,
                                     exchange=exchange, plan_splits=1)
        rows = plan.rows_of(rank)
        li, lo, fo = [], [], []
        for i, layer in enumerate(layers):
            hs = torch.tensor(plan.heads_of(rank, layer), device=dev)
            li.append([tuple(x[rows[0]:rows[-1] + 1].index_select(1, hs).contiguous()
                             for x in inputs[i][t]) for t in range(full.num_scales)])
            lo.append([torch.empty(plan.rows_per_rank, n, plan.heads_per_rank * 128, device=dev,
                                   dtype=torch.bfloat16) for n in full.tokens])
        fo, _flat = sh.allocate_full_outputs(batch, H)
        for row in fo:
            for x in row:
                x.fill_(float("nan"))
        torch.cuda.synchronize(dev)
        dist.barrier()   # peers store into this rank's outputs: fill them before anyone runs
        launches = sh.launches(li, lo, fo, sh.allocate_gather_buffer())
        stream = torch.cuda.Stream(dev)
        stream.wait_stream(torch.cuda.current_stream(dev))   # the inputs were made on it
        with torch.cuda.stream(stream):
            HotPath.run(launches, stream)
        stream.synchronize()

        def check(tag):
            good = True
            for i in range(len(layers)):
                for t in range(full.num_scales):
                    if not torch.equal(fo[i][t], ref_out[i][t]):
                        err = (fo[i][t].float() - ref_out[i][t].float()).abs().max().item()
                        print(f"rank {rank} {tag}: layer {layers[i]} target {t} differs "
                              f"(max {err})", flush=True)
                        good = False
            return good

        ok = check("eager") and ok
        if rank == 0:
            # the last layer of the pair (it has pruned targets) against the keep-mask semantics
            i = len(layers) - 1
            for t in range(full.num_scales):
                ref = keep_mask_attention(ctrl, layers[i], t, inputs[i])
                err = (fo[i][t].float() - ref).abs().max().item()
                scale = ref.abs().max().item()
                if not (err <= BF16_ATOL and err / scale <= BF16_REL):
                    print(f"rank 0: layer {layers[i]} target {t} vs keep-mask attention: max "
                          f"{err} (scale {scale})", flush=True)
                    ok = False
        for row in fo:
            for x in row:
                x.fill_(float("nan"))
        torch.cuda.synchronize(dev)
        dist.barrier()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            HotPath.run(launches, stream)
        g.replay()
        torch.cuda.synchronize(dev)
        ok = check("graph") and ok
        del g
        torch.cuda.synchronize(dev)
        dist.barrier()   # no rank unmaps its peers' outputs while another still writes
        flags = _native.device_status(dev)
        if flags:
            print(f"rank {rank}: device flags {flags:#x}", flush=True)
            ok = False
        res = torch.tensor([0 if ok else 1], device=dev)
        dist.all_reduce(res)
        ok = res.item() == 0
        sh.close()
        if rank == 0:
            print(f"multi-GPU parity {'ok' if ok else 'FAILED'}: world {world}, split {split}, "
                  f"exchange {exchange}, rows x heads groups {plan.row_groups} x "
                  f"{plan.head_groups}", flush=True)
    finally:
        dist.destroy_process_group()
    return 0 if ok else 1


if __name__ == "__main__":
    sys.exit(main())
