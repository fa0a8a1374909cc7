"""The projection-driven hot path (random-init Infinity-2B QKV weights
driving Q/K/V) on the GPU.

* Against attention over exactly the tokens the keep-mask retains, in PyTorch fp32, on q/k/v from
  the PyTorch chain of the reference's forward (F.linear, F.normalize * scale_mul, apply_rotary_emb
  in fp32, q/k rounded to bf16 as the flash path's ``q.to(v.dtype)``): bf16 tolerance.
* Against the same preparation and the single-call engine run separately (``prepare_qkv`` for every
  (layer, scale), then ``HotPath`` with its own appends): outputs and slabs bit-identical, i.e. the
  early appends of the preparation leave the slab exactly as the reference's order does.
* The 64-row configuration: its first rows equal a 4-row run of the same rows (the rows of a
  batch are independent; only the projection GEMM may pick another algorithm at another size).
"""

import pytest
import torch
import torch.nn.functional as F

from heatkv_b200 import _native, synthetic
from heatkv_b200.hotpath import HotPath
from heatkv_b200.projected import ProjectedHotPath
from heatkv_b200.qkv_prep import prepare_qkv

from _keepmask import keep_mask_attention

pytestmark = pytest.mark.gpu

BF16_ATOL, BF16_REL = 2e-2, 1e-2


def _controller():
    import bench
    return bench.build_controller("2b", 0.10)


def _chain_qkv(x_t, w, start, n, cos, sin, scale_mul=4.0, heads=16):
    """The reference forward's chain for one scale (basic.py:282-292, :97-117), fp32 after the
    projection, q/k rounded to bf16 at the end."""
    B = x_t.shape[0]
    qkv = torch.mm(x_t.reshape(B * n, -1), w.t()).view(B, n, 3, heads, 128)
    q, k, v = qkv.permute(2, 0, 3, 1, 4).unbind(0)
    q = F.normalize(q.float(), dim=-1, eps=1e-12) * scale_mul
    k = F.normalize(k.float(), dim=-1, eps=1e-12)
    c, s = cos[start:start + n], sin[start:start + n]

    def rope(a):
        a = a.reshape(*a.shape[:-1], -1, 2)
        return torch.stack([c * a[..., 0] - s * a[..., 1], s * a[..., 0] + c * a[..., 1]],
                           dim=-1).reshape(*a.shape[:-2], -1)
    return rope(q).bfloat16(), rope(k).bfloat16(), v.contiguous()


def _run(ctrl, L, H, rows, layers, dev, row_ids=None, fused=True):
    hot = HotPath(ctrl, L, H, rows, dev, layers=layers)
    proj = ProjectedHotPath(hot, fused_projection=fused)
    x, _ = proj.allocate_inputs(row_ids if row_ids is not None else list(range(rows)), seed=3)
    outs = [proj.allocate_outputs()[0] for _ in layers]
    proj.run(proj.launches(x, outs))
    torch.cuda.synchronize(dev)
    return hot, proj, x, outs


@pytest.mark.parametrize("fused", [True, False])
def test_projected_path_matches_keep_mask_attention(fused):
    torch.backends.cuda.matmul.allow_tf32 = False
    dev = torch.device("cuda", 0)
    ctrl, L, H = _controller()
    layers = [0, 21]
    hot, proj, x, outs = _run(ctrl, L, H, 4, layers, dev, fused=fused)
    assert _native.device_status(dev) == 0
    assert proj.early_slots > 0 and proj.rest_slots > 0
    for i, layer in enumerate(layers):
        inputs = [_chain_qkv(x[t], proj.weights[i], proj.starts[t], proj.tokens[t],
                             proj.rope_cos, proj.rope_sin) for t in range(proj.num_scales)]
        for t in range(proj.num_scales):
            ref = keep_mask_attention(ctrl, layer, t, inputs, softmax_scale=1.0)
            err = (outs[i][t].float() - ref).abs().max().item()
            scale = ref.abs().max().item()
            assert err <= BF16_ATOL and err / scale <= BF16_REL, (layer, t, err, scale)


def test_projected_path_equals_prepare_then_hot_path():
    """Unfused projection (cuBLAS + heatkv_qkv_prepare_append): bit-identical to the preparation
    and the engine run separately."""
    dev = torch.device("cuda", 0)
    ctrl, L, H = _controller()
    layers = [3, 30]
    hot, proj, x, outs = _run(ctrl, L, H, 2, layers, dev, fused=False)
    # the same preparation per (layer, scale), then the engine with its own appends
    ref_hot = HotPath(ctrl, L, H, 2, dev, layers=layers)
    inputs, ref_out = [], []
    for i in range(len(layers)):
        row_in, row_out = [], []
        for t in range(proj.num_scales):
            n = proj.tokens[t]
            qkv = torch.mm(x[t].reshape(2 * n, -1), proj.weights[i].t()).view(2, n, 3, H, 128)
            c = proj.rope_cos[proj.starts[t]:proj.starts[t] + n]
            s = proj.rope_sin[proj.starts[t]:proj.starts[t] + n]
            row_in.append(prepare_qkv(qkv, scale_mul=proj.scale_mul, rope=(c, s),
                                      qk_dtype=torch.bfloat16))
            row_out.append(torch.empty(2, n, H * 128, dtype=torch.bfloat16, device=dev))
        inputs.append(row_in)
        ref_out.append(row_out)
    HotPath.run(ref_hot.launches(inputs, ref_out, softmax_scale=1.0))
    torch.cuda.synchronize(dev)
    assert _native.device_status(dev) == 0
    for i in range(len(layers)):
        for t in range(proj.num_scales):
            assert torch.equal(outs[i][t], ref_out[i][t]), (layers[i], t)
        # every live segment of the slab after the step (the last scale is never cached)
        p = hot.plans[i]
        for seg in p.schedule["segments"]:
            if seg["end_target"] < proj.num_scales:
                continue
            lo, hi = seg["offset"], seg["offset"] + seg["length"]
            assert torch.equal(hot.slab_k[i][:, lo:hi], ref_hot.slab_k[i][:, lo:hi]), seg
            assert torch.equal(hot.slab_v[i][:, lo:hi], ref_hot.slab_v[i][:, lo:hi]), seg


def test_projected_64_rows_match_4_rows():
    """configs[4] size (64 rows) on two layers: rows 0..3 agree with a 4-row run of the same rows;
    rows 60..63 with a 4-row run of those rows."""
    dev = torch.device("cuda", 0)
    ctrl, L, H = _controller()
    layers = [0, 21]
    _, big, _, out64 = _run(ctrl, L, H, 64, layers, dev)
    assert _native.device_status(dev) == 0
    for ids, sl in (([0, 1, 2, 3], slice(0, 4)), ([60, 61, 62, 63], slice(60, 64))):
        _, _, _, out4 = _run(ctrl, L, H, 4, layers, dev, row_ids=ids)
        for i in range(len(layers)):
            for t in range(big.num_scales):
                a, b = out64[i][t][sl].float(), out4[i][t].float()
                err = (a - b).abs().max().item()
                assert err <= BF16_ATOL and err / max(b.abs().max().item(), 1e-6) <= BF16_REL, \
                    (layers[i], t, err)


def test_fused_projection_path_matches_unfused_path():
    """The fused projection (tcgen05 GEMM with the preparation and early appends in its epilogue)
    against the unfused path on the same rows: every output and every live slab segment after the
    step within the bf16 tolerance."""
    dev = torch.device("cuda", 0)
    ctrl, L, H = _controller()
    layers = [0, 17]
    runs = [_run(ctrl, L, H, 4, layers, dev, fused=f) for f in (True, False)]
    assert _native.device_status(dev) == 0
    (ha, _, _, oa), (hb, _, _, ob) = runs
    for i in range(len(layers)):
        for a, b in zip(oa[i], ob[i]):
            err = (a.float() - b.float()).abs().max().item()
            assert err <= BF16_ATOL and err <= BF16_REL * b.float().abs().max().item(), err
        for seg in ha.plans[i].schedule["segments"]:
            if seg["end_target"] < ha.num_scales:
                continue
            lo, hi = seg["offset"], seg["offset"] + seg["length"]
            for sa, sb in ((ha.slab_k[i], hb.slab_k[i]), (ha.slab_v[i], hb.slab_v[i])):
                err = (sa[:, lo:hi].float() - sb[:, lo:hi].float()).abs().max().item()
                assert err <= BF16_ATOL, (seg, err)
