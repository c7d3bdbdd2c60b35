"""Differential tests: every sm_100a kernel against its fp32 PyTorch contract (ops/reference.py)."""

import math

import pytest
import torch

from inference_systems_b200 import ops
from inference_systems_b200.ops import reference as ref

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(scope="module", autouse=True)
def _load_kernels():
    ops.cuda_ops()  # registers torch.ops.isb.* before tests call them directly


def _rel(a, b):
    a, b = a.float().cpu(), b.float().cpu()
    return ((a - b).norm() / (b.norm() + 1e-12)).item()


@pytest.fixture(autouse=True)
def _no_device_errors():
    yield
    torch.cuda.synchronize()
    assert ops.cuda_ops().error_word() == 0, "a kernel recorded a bounded-wait timeout"


@pytest.mark.parametrize("m,n,k", [(1, 8224, 1024), (5, 1024, 2048), (16, 2048, 1024), (37, 7168, 1024),
                                   (64, 1024, 3584), (128, 4096, 1024), (129, 1024, 1024), (300, 8224, 1024),
                                   (1000, 1024, 2048), (2048, 7168, 1024)])
def test_gemm(m, n, k):
    g = torch.Generator(device=DEV).manual_seed(m * 7 + n)
    a = torch.randn(m, k, device=DEV, generator=g).to(torch.bfloat16)
    b = (torch.randn(n, k, device=DEV, generator=g) * 0.05).to(torch.bfloat16)
    out = ops.linear(a, b)
    exp = a.float() @ b.float().t()
    assert out.shape == (m, n)
    assert _rel(out, exp) < 1e-2


@pytest.mark.parametrize("m,inter,k", [(1, 3584, 1024), (8, 1792, 1024), (96, 448, 1024), (200, 3584, 1024),
                                       (512, 896, 1024)])
def test_gemm_silu_mul(m, inter, k):
    g = torch.Generator(device=DEV).manual_seed(m + inter)
    a = torch.randn(m, k, device=DEV, generator=g).to(torch.bfloat16)
    gate = (torch.randn(inter, k, device=DEV, generator=g) * 0.05).to(torch.bfloat16)
    up = (torch.randn(inter, k, device=DEV, generator=g) * 0.05).to(torch.bfloat16)
    w = ref.pack_gate_up(gate, up)
    out = ops.linear_silu_mul(a, w)
    exp = torch.nn.functional.silu(a.float() @ gate.float().t()) * (a.float() @ up.float().t())
    assert out.shape == (m, inter)
    assert _rel(out, exp) < 1e-2


@pytest.mark.parametrize("b,v", [(1, 248320), (7, 4096), (64, 248320), (160, 32768)])
def test_lm_head_greedy(b, v):
    g = torch.Generator(device=DEV).manual_seed(b)
    h = torch.randn(b, 1024, device=DEV, generator=g).to(torch.bfloat16)
    w = (torch.randn(v, 1024, device=DEV, generator=g) * 0.05).to(torch.bfloat16)
    temps = torch.zeros(b, device=DEV)
    rng = torch.tensor([0, 0], dtype=torch.int32, device=DEV)
    val, idx = ops.lm_head_sample(h, w, temps, rng, 0)
    logits = h.float() @ w.float().t()
    best = logits.max(-1).values
    picked = logits.gather(1, idx.long()[:, None]).squeeze(1)
    assert torch.all(best - picked < 2e-2 * best.abs().clamp(min=1)), (best - picked).max()


def test_lm_head_gumbel_matches_host_noise():
    g = torch.Generator(device=DEV).manual_seed(3)
    b, v = 4, 4096
    h = torch.randn(b, 256, device=DEV, generator=g).to(torch.bfloat16)
    w = (torch.randn(v, 256, device=DEV, generator=g) * 0.5).to(torch.bfloat16)
    temps = torch.tensor([0.0, 0.7, 1.0, 1.5], device=DEV)
    rng = torch.tensor([1234, 17], dtype=torch.int32, device=DEV)
    _, idx = ops.lm_head_sample(h, w, temps, rng, 0)
    logits = (h.float() @ w.float().t())
    _, exp_idx = ops.gumbel_select(logits.cpu(), temps.cpu(), 1234, 17, 0)
    assert (idx.cpu().long() == exp_idx).float().mean() >= 0.75


@pytest.mark.parametrize("rows,h,zc", [(1, 1024, True), (37, 1024, True), (128, 5120, True), (9, 1024, False)])
def test_norms(rows, h, zc):
    x = torch.randn(rows, h, device=DEV).to(torch.bfloat16)
    r = torch.randn(rows, h, device=DEV).to(torch.bfloat16)
    w = (torch.randn(h, device=DEV) * 0.1).to(torch.bfloat16)
    assert _rel(ops.rmsnorm(x, w, 1e-6, zc), ref.rmsnorm(x.cpu(), w.cpu(), 1e-6, zc)) < 1e-2
    r_gpu, r_cpu = r.clone(), r.cpu().clone()
    y = ops.add_rmsnorm(x, r_gpu, w, 1e-6, zc)
    y_ref = ref.add_rmsnorm(x.cpu(), r_cpu, w.cpu(), 1e-6, zc)
    assert _rel(y, y_ref) < 1e-2
    assert torch.equal(r_gpu.cpu(), r_cpu)


def test_embed():
    table = torch.randn(1000, 512, device=DEV).to(torch.bfloat16)
    ids = torch.randint(0, 1000, (33,), device=DEV, dtype=torch.int32)
    assert torch.equal(ops.embed(ids, table, 0), table[ids.long()])


def _gdn_inputs(b, hk, hv, seed, t=None):
    g = torch.Generator().manual_seed(seed)
    d = 128
    c = 2 * hk * d + hv * d
    p = c + hv * d + 2 * hv
    t = t or b
    proj = (torch.randn(t, p, generator=g)).to(torch.bfloat16)
    conv_w = (torch.randn(c, 4, generator=g) * 0.5).to(torch.bfloat16)
    a_log = torch.randn(hv, generator=g) * 0.5
    dt_bias = torch.randn(hv, generator=g) * 0.5
    norm_w = (1 + 0.1 * torch.randn(d, generator=g)).to(torch.bfloat16)
    slots = 3 * b + 2
    rec = torch.randn(slots, hv, d, d, generator=g) * 0.1
    conv = torch.randn(slots, c, 3, generator=g).to(torch.bfloat16)
    slot_ids = torch.randperm(slots, generator=g)[:b].to(torch.int32)
    return proj, conv_w, a_log, dt_bias, norm_w, rec, conv, slot_ids


@pytest.mark.parametrize("b,hk,hv", [(1, 16, 16), (7, 16, 16), (64, 4, 4), (5, 2, 6), (48, 16, 16), (320, 2, 6)])
def test_gdn_decode(b, hk, hv):
    proj, conv_w, a_log, dt_bias, norm_w, rec, conv, slots = _gdn_inputs(b, hk, hv, b + hk)
    rec_c, conv_c = rec.clone(), conv.clone()
    cu = list(range(b + 1))
    exp = ref.gdn_forward(proj, cu, slots.tolist(), conv_w, a_log, dt_bias, norm_w, rec_c, conv_c,
                          hk=hk, hv=hv, dk=128, dv=128, eps=1e-6)
    rec_g, conv_g = rec.to(DEV), conv.to(DEV)
    proj_acc = proj.float().to(DEV)  # fp32 accumulator input, consumed by the kernel
    out = torch.ops.isb.gdn_decode(proj_acc, slots.to(DEV), conv_w.to(DEV), a_log.to(DEV), dt_bias.to(DEV),
                                   norm_w.to(DEV), rec_g, conv_g, hk, hv, 128, 128, 1e-6)
    assert torch.count_nonzero(proj_acc) == 0
    assert _rel(out.cpu(), exp) < 2e-2
    assert _rel(rec_g.cpu(), rec_c) < 1e-4
    assert torch.equal(conv_g.cpu(), conv_c)


@pytest.mark.parametrize("lens,hk,hv", [([5, 1, 33], 16, 16), ([64, 17], 2, 6), ([300], 4, 4)])
def test_gdn_prefill(lens, hk, hv):
    b, t = len(lens), sum(lens)
    proj, conv_w, a_log, dt_bias, norm_w, rec, conv, slots = _gdn_inputs(b, hk, hv, t, t=t)
    cu = [0]
    for n in lens:
        cu.append(cu[-1] + n)
    rec_c, conv_c = rec.clone(), conv.clone()
    exp = ref.gdn_forward(proj, cu, slots.tolist(), conv_w, a_log, dt_bias, norm_w, rec_c, conv_c,
                          hk=hk, hv=hv, dk=128, dv=128, eps=1e-6)
    rec_g, conv_g = rec.to(DEV), conv.to(DEV)
    out = torch.ops.isb.gdn_prefill(proj.to(DEV), torch.tensor(cu, dtype=torch.int32, device=DEV), slots.to(DEV),
                                    conv_w.to(DEV), a_log.to(DEV), dt_bias.to(DEV), norm_w.to(DEV), rec_g, conv_g,
                                    hk, hv, 128, 128, 1e-6, max(lens))
    assert _rel(out.cpu(), exp) < 2e-2
    assert _rel(rec_g.cpu(), rec_c) < 1e-3
    assert torch.equal(conv_g.cpu(), conv_c)


@pytest.mark.parametrize("lens,hk,hv", [([5, 1, 33], 16, 16), ([64, 65, 17], 2, 6), ([300, 128], 4, 4),
                                         ([1000], 2, 4)])
def test_gdn_prefill_chunked_matches_scan_and_oracle(lens, hk, hv):
    from inference_systems_b200.ops import GDN_CHUNK

    b, t = len(lens), sum(lens)
    proj, conv_w, a_log, dt_bias, norm_w, rec, conv, slots = _gdn_inputs(b, hk, hv, t, t=t)
    cu = [0]
    for n in lens:
        cu.append(cu[-1] + n)
    rec_c, conv_c = rec.clone(), conv.clone()
    exp = ref.gdn_forward(proj, cu, slots.tolist(), conv_w, a_log, dt_bias, norm_w, rec_c, conv_c,
                          hk=hk, hv=hv, dk=128, dv=128, eps=1e-6)
    seq, t0, nn, cuc = [], [], [], [0]
    for i in range(b):
        for st in range(cu[i], cu[i + 1], GDN_CHUNK):
            seq.append(i)
            t0.append(st)
            nn.append(min(GDN_CHUNK, cu[i + 1] - st))
        cuc.append(len(seq))
    info = torch.tensor(seq + t0 + nn + cuc, dtype=torch.int32, device=DEV)
    args = (conv_w.to(DEV), a_log.to(DEV), dt_bias.to(DEV), norm_w.to(DEV))
    cu_d = torch.tensor(cu, dtype=torch.int32, device=DEV)
    rec_k, conv_k = rec.to(DEV), conv.to(DEV)
    out_k = torch.ops.isb.gdn_prefill_chunked(proj.to(DEV), cu_d, slots.to(DEV), info, len(seq), *args, rec_k, conv_k,
                                              hk, hv, 1e-6)
    rec_s, conv_s = rec.to(DEV), conv.to(DEV)
    out_s = torch.ops.isb.gdn_prefill(proj.to(DEV), cu_d, slots.to(DEV), *args, rec_s, conv_s, hk, hv, 128, 128,
                                      1e-6, max(lens))
    torch.cuda.synchronize()
    assert _rel(out_k.cpu(), exp) < 2e-2
    assert _rel(out_k.float(), out_s.float()) < 2e-2
    assert _rel(rec_k.cpu(), rec_c) < 1e-3
    assert _rel(rec_k, rec_s) < 1e-3
    assert torch.equal(conv_k.cpu(), conv_c)


@pytest.mark.parametrize("lens,hk,hv,marks", [([300, 40], 16, 16, [[99, 255], [9]]), ([130], 2, 4, [[0, 64, 129]])])
def test_gdn_scan_history_states_match_oracle(lens, hk, hv, marks):
    b, t = len(lens), sum(lens)
    proj, conv_w, a_log, dt_bias, norm_w, rec, conv, slots = _gdn_inputs(b, hk, hv, 7 * t, t=t)
    cu = [0]
    for n in lens:
        cu.append(cu[-1] + n)
    rows = [-1] * t
    k = 0
    for i, ms in enumerate(marks):
        for m in ms:
            rows[cu[i] + m] = k
            k += 1
    hist_rec_r, hist_conv_r = [None] * k, [None] * k
    rec_c, conv_c = rec.clone(), conv.clone()
    for i in range(b):
        _, r_fin, c_fin, rh, ch, _ = ref.gdn_sequence(proj[cu[i]:cu[i + 1]], conv_w, a_log, dt_bias, norm_w,
                                                      rec_c[slots[i]], conv_c[slots[i]], hk=hk, hv=hv, dk=128, dv=128,
                                                      eps=1e-6, history_at=marks[i])
        for m, rs_, cs_ in zip(marks[i], rh, ch):
            hist_rec_r[rows[cu[i] + m]] = rs_
            hist_conv_r[rows[cu[i] + m]] = cs_
    c = 2 * hk * 128 + hv * 128
    hist_rec = torch.zeros(k, hv, 128, 128, device=DEV)
    hist_conv = torch.zeros(k, c, 3, device=DEV, dtype=torch.bfloat16)
    rec_g, conv_g = rec.to(DEV), conv.to(DEV)
    torch.ops.isb.gdn_scan_history(proj.to(DEV), torch.tensor(cu, dtype=torch.int32, device=DEV), slots.to(DEV),
                                   conv_w.to(DEV), a_log.to(DEV), dt_bias.to(DEV), norm_w.to(DEV), rec_g, conv_g,
                                   hk, hv, 1e-6, True, torch.tensor(rows, dtype=torch.int32, device=DEV), hist_rec,
                                   hist_conv, None, None, None)
    torch.cuda.synchronize()
    for j in range(k):
        assert _rel(hist_rec[j].cpu(), hist_rec_r[j]) < 1e-3, j
        assert torch.equal(hist_conv[j].cpu(), hist_conv_r[j].to(torch.bfloat16)), j


def gate_ref(qkv, hq, hd):
    t = qkv.shape[0]
    return qkv[:, : hq * hd * 2].reshape(t, hq, 2 * hd)[..., hd:].reshape(t, hq * hd)


def _attn_case(seed, hq, hkv, hd, lens_new, lens_past, gated=True, fill=0.0, nblocks=64, mb=8):
    g = torch.Generator().manual_seed(seed)
    b = len(lens_new)
    kc = torch.full((nblocks, hkv, 256, hd), fill, dtype=torch.bfloat16)
    vc = torch.full_like(kc, fill)
    perm = torch.randperm(nblocks, generator=g)
    bt = torch.full((b, mb), -1, dtype=torch.int32)
    ids, pos, slots, cu, ctx = [], [], [], [0], []
    used = 0
    for i, (n, past) in enumerate(zip(lens_new, lens_past)):
        total = n + past
        nb = (total + 255) // 256
        bt[i, :nb] = perm[used:used + nb].to(torch.int32)
        used += nb
        for p in range(past, total):
            pos.append(p)
            slots.append(int(bt[i, p // 256]) * 256 + p % 256)
        cu.append(cu[-1] + n)
        ctx.append(total)
        # pre-fill the cached prefix rows with random K/V
        for p in range(past):
            kc[bt[i, p // 256], :, p % 256] = torch.randn(hkv, hd, generator=g).to(torch.bfloat16)
            vc[bt[i, p // 256], :, p % 256] = torch.randn(hkv, hd, generator=g).to(torch.bfloat16)
    t = cu[-1]
    width = hq * hd * (2 if gated else 1) + 2 * hkv * hd
    qkv = torch.randn(t, width, generator=g).to(torch.bfloat16)
    qn = (0.1 * torch.randn(hd, generator=g)).to(torch.bfloat16)
    kn = (0.1 * torch.randn(hd, generator=g)).to(torch.bfloat16)
    cos_sin = ref.rope_cos_sin(4096, hd // 4, 1e7)
    meta = dict(positions=torch.tensor(pos, dtype=torch.int32), slot_mapping=torch.tensor(slots, dtype=torch.int32),
                cu=torch.tensor(cu, dtype=torch.int32), ctx=torch.tensor(ctx, dtype=torch.int32), bt=bt)
    return qkv, qn, kn, cos_sin, kc, vc, meta


@pytest.mark.parametrize("hq,hkv,new,past", [(8, 2, [7, 1, 40], [0, 5, 300]), (4, 1, [257], [0]),
                                              (6, 1, [16, 3], [512, 0]), (2, 1, [33], [100])])
def test_attention_prefill(hq, hkv, new, past):
    hd = 256
    qkv, qn, kn, cos_sin, kc, vc, m = _attn_case(hq + sum(new), hq, hkv, hd, new, past)
    q, gate, k, v = ref.attn_qkv_prepare(qkv, m["positions"], qn, kn, cos_sin, hq, hkv, hd, 1e-6, True, True)
    kc_r, vc_r = kc.clone(), vc.clone()
    ref.store_kv(k, v, kc_r, vc_r, m["slot_mapping"])
    exp = ref.paged_attention(q, kc_r, vc_r, m["cu"], m["ctx"], m["bt"], hd ** -0.5, gate)
    kc_g, vc_g = kc.to(DEV), vc.to(DEV)
    qg, gate = torch.ops.isb.attn_prepare(qkv.to(DEV), m["positions"].to(DEV), m["slot_mapping"].to(DEV),
                                          qn.to(DEV), kn.to(DEV), cos_sin.to(DEV), kc_g, vc_g, hq, hkv, hd, 1e-6,
                                          True, True)
    assert _rel(qg.cpu(), q) < 1e-2
    assert _rel(gate.cpu(), gate_ref(qkv, hq, hd)) == 0
    assert _rel(kc_g.cpu(), kc_r) < 1e-2 and _rel(vc_g.cpu(), vc_r) < 1e-2
    out = torch.ops.isb.attention_prefill(qg, gate, kc_g, vc_g, m["cu"].to(DEV), m["ctx"].to(DEV),
                                          m["bt"].to(DEV), hd ** -0.5, True, max(new))
    assert _rel(out.cpu(), exp) < 2e-2


@pytest.mark.parametrize("hq,hkv,new,past", [(8, 2, [7, 1, 40], [0, 5, 300]), (8, 2, [300, 65], [0, 200]),
                                              (4, 1, [257], [0]), (2, 1, [130], [100]), (16, 2, [20, 9], [64, 0]),
                                              (6, 1, [100, 43], [0, 300]), (12, 4, [50], [10]), (3, 1, [90], [0])])
def test_attention_prefill_tensor_core(hq, hkv, new, past):
    hd = 256
    qkv, qn, kn, cos_sin, kc, vc, m = _attn_case(7 * hq + sum(new), hq, hkv, hd, new, past)
    q, gate, k, v = ref.attn_qkv_prepare(qkv, m["positions"], qn, kn, cos_sin, hq, hkv, hd, 1e-6, True, True)
    kc_r, vc_r = kc.clone(), vc.clone()
    ref.store_kv(k, v, kc_r, vc_r, m["slot_mapping"])
    exp = ref.paged_attention(q, kc_r, vc_r, m["cu"], m["ctx"], m["bt"], hd ** -0.5, gate)
    kc_g, vc_g = kc.to(DEV), vc.to(DEV)
    qg, gate_g = torch.ops.isb.attn_prepare(qkv.to(DEV), m["positions"].to(DEV), m["slot_mapping"].to(DEV),
                                            qn.to(DEV), kn.to(DEV), cos_sin.to(DEV), kc_g, vc_g, hq, hkv, hd, 1e-6,
                                            True, True)
    args = (qg, gate_g, kc_g, vc_g, m["cu"].to(DEV), m["ctx"].to(DEV), m["bt"].to(DEV), hd ** -0.5, True, max(new))
    out_tc = torch.ops.isb.attention_prefill_tc(*args)
    out_simt = torch.ops.isb.attention_prefill(*args)
    torch.cuda.synchronize()
    assert torch.ops.isb.error_word() == 0
    assert _rel(out_tc.cpu(), exp) < 2e-2
    assert _rel(out_tc.float(), out_simt.float()) < 2e-2


@pytest.mark.parametrize("hq,hkv,past", [(8, 2, [0, 5, 300, 1000]), (4, 1, [255]), (24, 4, [2000, 1]),
                                         (3, 1, [700])])
def test_attention_decode(hq, hkv, past):
    hd = 256
    new = [1] * len(past)
    qkv, qn, kn, cos_sin, kc, vc, m = _attn_case(hq + sum(past), hq, hkv, hd, new, past)
    q, gate, k, v = ref.attn_qkv_prepare(qkv, m["positions"], qn, kn, cos_sin, hq, hkv, hd, 1e-6, True, True)
    kc_r, vc_r = kc.clone(), vc.clone()
    ref.store_kv(k, v, kc_r, vc_r, m["slot_mapping"])
    exp = ref.paged_attention(q, kc_r, vc_r, m["cu"], m["ctx"], m["bt"], hd ** -0.5, gate)
    kc_g, vc_g = kc.to(DEV), vc.to(DEV)
    # fp32 accumulator input path: the prepare kernel consumes (re-zeroes) the projection
    qkv_acc = qkv.float().to(DEV)
    qg, gate = torch.ops.isb.attn_prepare(qkv_acc, m["positions"].to(DEV), m["slot_mapping"].to(DEV), qn.to(DEV),
                                          kn.to(DEV), cos_sin.to(DEV), kc_g, vc_g, hq, hkv, hd, 1e-6, True, True)
    assert torch.count_nonzero(qkv_acc) == 0
    out = torch.ops.isb.attention_decode(qg, gate, kc_g, vc_g, m["ctx"].to(DEV), m["bt"].to(DEV),
                                         hd ** -0.5, True)
    assert _rel(out.cpu(), exp) < 2e-2


@pytest.mark.parametrize("hq,hkv,past", [
    (8, 2, [0, 126, 127, 128, 129, 255, 256, 300, 511, 1000]),
    (24, 8, [2000, 1, 383]),      # G = 3
    (16, 2, [127, 700, 5]),       # G = 8
    (6, 1, [128, 129]),           # G = 6
    (2, 1, [40, 1500]),           # G = 2
    (4, 4, [257, 64]),            # G = 1
])
def test_attention_decode_tc(hq, hkv, past):
    """Tensor-core split-KV decode vs the fp32 reference and the SIMT kernel.  Cache rows
    that no sequence owns hold NaN: the last-tile masking must keep them out."""
    hd = 256
    new = [1] * len(past)
    qkv, qn, kn, cos_sin, kc, vc, m = _attn_case(7 * hq + sum(past), hq, hkv, hd, new, past, fill=float("nan"),
                                                 nblocks=48, mb=9)
    q, gate, k, v = ref.attn_qkv_prepare(qkv, m["positions"], qn, kn, cos_sin, hq, hkv, hd, 1e-6, True, True)
    kc_r, vc_r = kc.clone(), vc.clone()
    ref.store_kv(k, v, kc_r, vc_r, m["slot_mapping"])
    exp = ref.paged_attention(q, kc_r, vc_r, m["cu"], m["ctx"], m["bt"], hd ** -0.5, gate)
    assert torch.isfinite(exp).all()
    kc_g, vc_g = kc.to(DEV), vc.to(DEV)
    qg, gate_g = torch.ops.isb.attn_prepare(qkv.to(DEV), m["positions"].to(DEV), m["slot_mapping"].to(DEV),
                                            qn.to(DEV), kn.to(DEV), cos_sin.to(DEV), kc_g, vc_g, hq, hkv, hd, 1e-6,
                                            True, True)
    args = (qg, gate_g, kc_g, vc_g, m["ctx"].to(DEV), m["bt"].to(DEV), hd ** -0.5, True)
    out_tc = torch.ops.isb.attention_decode_tc(*args)
    torch.cuda.synchronize()
    assert torch.ops.isb.error_word() == 0
    assert torch.isfinite(out_tc.float()).all()
    assert _rel(out_tc.cpu(), exp) < 2e-2
    out_auto = torch.ops.isb.attention_decode(*args)
    assert _rel(out_auto.float(), out_tc.float()) < 2e-2


def test_state_int8_roundtrip_and_page_copy():
    x = torch.randn(3, 4, 128, 128, device=DEV)
    q = torch.empty(x.shape, dtype=torch.int8, device=DEV)
    s = torch.empty(3, 4, 128, 1, device=DEV)
    ops.quantize_state_int8(x, q, s)
    qc, sc = torch.empty(x.shape, dtype=torch.int8), torch.empty(3, 4, 128, 1)
    ops.quantize_state_int8(x.cpu(), qc, sc)
    assert torch.equal(q.cpu(), qc) and torch.allclose(s.cpu(), sc)
    out = torch.empty_like(x)
    ops.dequantize_state_int8(q, s, out)
    assert (out - x).abs().max() <= s.max() * 0.51
    kc = torch.randn(4, 2, 256, 256, device=DEV).to(torch.bfloat16)
    vc = torch.randn_like(kc)
    k0, v0 = kc.clone(), vc.clone()
    ops.copy_kv_page(kc, vc, 1, 3, 100)
    assert torch.equal(kc[3, :, :100], k0[1, :, :100]) and torch.equal(kc[3, :, 100:], k0[3, :, 100:])
    assert torch.equal(vc[3, :, :100], v0[1, :, :100])


@pytest.mark.parametrize("m,n,k", [(1, 1024, 2048), (37, 1024, 3584), (128, 1024, 2048), (300, 1024, 3584)])
def test_gemm_accumulate_and_norm(m, n, k):
    g = torch.Generator(device=DEV).manual_seed(m + k)
    a = torch.randn(m, k, device=DEV, generator=g).to(torch.bfloat16)
    b = (torch.randn(n, k, device=DEV, generator=g) * 0.05).to(torch.bfloat16)
    acc = torch.zeros(m + 3, n, device=DEV)
    ops.linear_accumulate(a, b, acc)
    exp = a.float() @ b.float().t()
    assert _rel(acc[:m], exp) < 1e-3
    assert torch.count_nonzero(acc[m:]) == 0
    resid = torch.randn(m, n, device=DEV).to(torch.bfloat16)
    w = (torch.randn(n, device=DEV) * 0.1).to(torch.bfloat16)
    r_ref = resid.cpu().clone()
    exp_out = ref.add_rmsnorm(exp.cpu(), r_ref, w.cpu(), 1e-6, True)
    out = ops.add_rmsnorm_acc(acc, resid, w, 1e-6, True)
    assert _rel(out, exp_out) < 1e-2
    assert _rel(resid, r_ref) < 1e-2
    assert torch.count_nonzero(acc) == 0, "consumer must re-zero the accumulator"


@pytest.mark.parametrize("m,n,k,zc", [(1, 1024, 2048, True), (37, 1024, 3584, False), (128, 1024, 2048, True),
                                      (128, 1024, 3584, True), (300, 1024, 3584, True), (96, 5120, 17408, True)])
def test_gemm_accum_norm_fused(m, n, k, zc):
    """One kernel: split-K accumulate, in-kernel grid barrier, residual add + RMSNorm (grids that
    fit on the SMs; larger ones take the two-kernel path).  Repeated calls cycle the barrier's
    counter slots, which must come back to zero."""
    g = torch.Generator(device=DEV).manual_seed(m + k + n)
    a = torch.randn(m, k, device=DEV, generator=g).to(torch.bfloat16)
    b = (torch.randn(n, k, device=DEV, generator=g) * 0.05).to(torch.bfloat16)
    w = (torch.randn(n, device=DEV, generator=g) * 0.1).to(torch.bfloat16)
    acc = torch.zeros(m + 3, n, device=DEV)
    exp = a.float() @ b.float().t()
    for it in range(10):
        resid = torch.randn(m, n, device=DEV, generator=g).to(torch.bfloat16)
        r_ref = resid.cpu().clone()
        exp_out = ref.add_rmsnorm(exp.cpu(), r_ref, w.cpu(), 1e-6, zc)
        out = ops.linear_add_rmsnorm(a, b, acc, resid, w, 1e-6, zc)
        assert _rel(out, exp_out) < 1e-2, it
        assert _rel(resid, r_ref) < 1e-2, it
        assert torch.count_nonzero(acc) == 0, "the fused tail must re-zero the accumulator"


def test_silu_mul_acc():
    acc = torch.randn(9, 2 * 448, device=DEV)
    exp = ref.silu_mul_packed(acc.cpu())
    out = ops.silu_mul_acc(acc, 7)
    assert _rel(out, exp[:7]) < 1e-2
    assert torch.count_nonzero(acc[:7]) == 0 and torch.count_nonzero(acc[7:]) > 0


def test_embed_rmsnorm():
    table = torch.randn(500, 1024, device=DEV).to(torch.bfloat16)
    w = (torch.randn(1024, device=DEV) * 0.1).to(torch.bfloat16)
    ids = torch.randint(0, 500, (17,), device=DEV, dtype=torch.int32)
    res, out = ops.embed_rmsnorm(ids, table, w, 1e-6, True)
    assert torch.equal(res, table[ids.long()])
    assert _rel(out, ref.rmsnorm(table[ids.long()].cpu(), w.cpu(), 1e-6, True)) < 1e-2
