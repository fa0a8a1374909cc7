"""One rank of the multi-GPU check of the benchmark workload (launched by test_gpu_multi.py under
torchrun): BASELINE configs[4]'s projection-driven hot path with the batch sharded by rows.

Every rank plans the same (row, head) shards (``sharding.plan_shards``, rows only: each row's
outputs are used on the GPU that computed them), generates its rows' layer inputs from the per-row
seeds, runs two 2B layers over all 13 scales, and the ranks all-gather their attention outputs to
rank 0 over NCCL. Rank 0 runs the whole batch on one GPU and requires the gathered outputs to be
bit-identical (every row's arithmetic is independent of the other rows), and checks one layer
against attention over exactly the tokens the keep-mask retains at the bf16 tolerance. Exit
status 0 = parity.
"""

import datetime
import os
import sys

import torch
import torch.distributed as dist
import torch.nn.functional as F

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
sys.path.insert(0, REPO)
sys.path.insert(0, HERE)

import bench  # noqa: E402
from heatkv_b200 import _native, sharding  # noqa: E402
from heatkv_b200.hotpath import HotPath  # noqa: E402
from heatkv_b200.projected import ProjectedHotPath  # noqa: E402
from _keepmask import keep_mask_attention  # noqa: E402

BF16_ATOL, BF16_REL = 2e-2, 1e-2


def run(ctrl, L, H, rows, layers, dev, row_ids):
    hot = HotPath(ctrl, L, H, rows, dev, layers=layers)
    proj = ProjectedHotPath(hot)
    x, _ = proj.allocate_inputs(row_ids, seed=5)
    outs = [proj.allocate_outputs()[0] for _ in layers]
    proj.run(proj.launches(x, outs))
    torch.cuda.synchronize(dev)
    return proj, x, outs


def chain_qkv(x_t, w, start, n, cos, sin):
    B = x_t.shape[0]
    qkv = torch.mm(x_t.reshape(B * n, -1), w.t()).view(B, n, 3, -1, 128)
    q, k, v = qkv.permute(2, 0, 3, 1, 4).unbind(0)
    q = F.normalize(q.float(), dim=-1, eps=1e-12) * 4.0
    k = F.normalize(k.float(), dim=-1, eps=1e-12)
    c, s = cos[start:start + n], sin[start:start + n]

    def rope(a):
        a = a.reshape(*a.shape[:-1], -1, 2)
        return torch.stack([c * a[..., 0] - s * a[..., 1], s * a[..., 0] + c * a[..., 1]],
                           dim=-1).reshape(*a.shape[:-2], -1)
    return rope(q).bfloat16(), rope(k).bfloat16(), v.contiguous()


def main() -> int:
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    ok = True
    try:
        ctrl, L, H = bench.build_controller("2b", 0.10)
        layers, batch = [0, 21], 2 * world
        plan = sharding.plan_shards(sharding.head_costs(ctrl, L, H), batch, world)
        assert not plan.splits_heads and plan.rows_per_rank == 2
        proj, _, outs = run(ctrl, L, H, plan.rows_per_rank, layers, dev, plan.rows_of(rank))
        flags = _native.device_status(dev)
        if flags:
            print(f"rank {rank}: device flags {flags:#x}", flush=True)
            ok = False
        gathered = []
        for i in range(len(layers)):
            row = []
            for t in range(proj.num_scales):
                o = outs[i][t].contiguous()
                buf = torch.empty((world,) + tuple(o.shape), dtype=o.dtype, device=dev)
                dist.all_gather_into_tensor(buf, o)
                row.append(buf.reshape(world * o.shape[0], *o.shape[1:]))
            gathered.append(row)
        if rank == 0:
            full, x, ref = run(ctrl, L, H, batch, layers, dev, list(range(batch)))
            order = plan.row_map().tolist()          # global row of each gathered row
            for i in range(len(layers)):
                for t in range(full.num_scales):
                    g = torch.empty_like(ref[i][t])
                    g[order] = gathered[i][t]
                    if not torch.equal(g, ref[i][t]):
                        err = (g.float() - ref[i][t].float()).abs().max().item()
                        print(f"rank 0: layer {layers[i]} target {t} differs from one GPU "
                              f"(max {err})", flush=True)
                        ok = False
            i = len(layers) - 1
            inputs = [chain_qkv(x[t], full.weights[i], full.starts[t], full.tokens[t],
                                full.rope_cos, full.rope_sin) for t in range(full.num_scales)]
            for t in range(full.num_scales):
                r = keep_mask_attention(ctrl, layers[i], t, inputs, softmax_scale=1.0)
                err = (ref[i][t].float() - r).abs().max().item()
                scale = r.abs().max().item()
                if not (err <= BF16_ATOL and err / scale <= BF16_REL):
                    print(f"rank 0: layer {layers[i]} target {t} vs keep-mask attention: max "
                          f"{err} (scale {scale})", flush=True)
                    ok = False
        res = torch.tensor([0 if ok else 1], device=dev)
        dist.all_reduce(res)
        ok = res.item() == 0
        if rank == 0:
            print(f"projected multi-GPU parity {'ok' if ok else 'FAILED'}: world {world}, rows "
                  f"{batch}, row groups {plan.row_groups}", flush=True)
    finally:
        dist.destroy_process_group()
    return 0 if ok else 1


if __name__ == "__main__":
    sys.exit(main())
