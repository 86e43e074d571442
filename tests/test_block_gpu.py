"""The GDN block on B200 (recant_b200.block) against the reference's eager CPU ops stage by stage
and against the reference block (golden output) / the block oracle (gradients) end to end."""
import pytest
import torch
import torch.nn.functional as F

from block_util import HIDDEN, HK, HV, golden, oracle_params
from gpu_util import rel
from oracle import block as OB

pytestmark = pytest.mark.gpu


def test_conv_silu_split_forward_backward():
    from recant_b200.block import conv_silu
    gen = torch.Generator().manual_seed(3)
    B, T, C, s1, s2 = 2, 100, 512, 128, 256
    x = torch.randn(B, T, C, generator=gen).to(torch.bfloat16)
    w = (torch.randn(C, 1, 4, generator=gen) * 0.4).to(torch.bfloat16)
    dy = torch.randn(B, T, C, generator=gen).to(torch.bfloat16)
    # reference eager path (layers.py:162-166) with autograd on the CPU
    xr = x.clone().requires_grad_(True)
    cat = torch.cat([torch.zeros(B, C, 3, dtype=torch.bfloat16), xr.transpose(1, 2)], -1)
    ref = F.silu(F.conv1d(cat, w, groups=C)).transpose(1, 2)
    ref.backward(dy)
    xd = x.cuda().requires_grad_(True)
    q, k, v = conv_silu(xd, w.cuda(), s1, s2)
    out = torch.cat([q, k, v], -1)
    out.backward(dy.cuda())
    torch.cuda.synchronize()
    assert rel(out.float(), ref.float()) < 1e-2
    assert rel(xd.grad.float(), xr.grad.float()) < 1e-2


def test_gates_forward_backward():
    from recant_b200.block import gdn_gates
    gen = torch.Generator().manual_seed(4)
    a = (torch.randn(3, 50, 8, generator=gen) * 4).to(torch.bfloat16)
    b = torch.randn(3, 50, 8, generator=gen).to(torch.bfloat16)
    A_log = torch.log(torch.empty(8).uniform_(1, 16, generator=gen))
    dt_bias = torch.randn(8, generator=gen)
    dg, db = torch.randn(3, 50, 8, generator=gen), torch.randn(3, 50, 8, generator=gen).to(torch.bfloat16)
    ar, br = a.clone().requires_grad_(True), b.clone().requires_grad_(True)
    g_ref = -A_log.exp() * F.softplus(ar.float() + dt_bias)      # fused_ops.py:32-33
    beta_ref = br.sigmoid()
    (g_ref * dg).sum().backward(retain_graph=True)
    beta_ref.backward(db)
    ad, bd = a.cuda().requires_grad_(True), b.cuda().requires_grad_(True)
    g, beta = gdn_gates(ad, bd, A_log.cuda(), dt_bias.cuda())
    (g * dg.cuda()).sum().backward(retain_graph=True)
    beta.backward(db.cuda())
    assert rel(g, g_ref) < 1e-5 and rel(beta.float(), beta_ref.float()) < 1e-2
    assert rel(ad.grad.float(), ar.grad.float()) < 1e-2 and rel(bd.grad.float(), br.grad.float()) < 1e-2


def test_gated_rmsnorm_forward_backward():
    from recant_b200.block import gated_rmsnorm
    gen = torch.Generator().manual_seed(5)
    x = torch.randn(300, 128, generator=gen).to(torch.bfloat16)
    z = torch.randn(300, 128, generator=gen).to(torch.bfloat16)
    w = (1 + 0.1 * torch.randn(128, generator=gen)).to(torch.bfloat16)
    dy = torch.randn(300, 128, generator=gen).to(torch.bfloat16)
    xr, zr = x.clone().requires_grad_(True), z.clone().requires_grad_(True)
    y = xr.float()
    y = y * torch.rsqrt(y.pow(2).mean(-1, keepdim=True) + 1e-6)   # fused_ops.py:11-16
    y = w * y.to(torch.bfloat16)
    ref = (y * F.silu(zr.float())).to(torch.bfloat16)
    ref.backward(dy)
    xd, zd = x.cuda().requires_grad_(True), z.cuda().requires_grad_(True)
    out = gated_rmsnorm(xd, zd, w.cuda().float())
    out.backward(dy.cuda())
    assert rel(out.float(), ref.float()) < 1e-2
    assert rel(xd.grad.float(), xr.grad.float()) < 2e-2 and rel(zd.grad.float(), zr.grad.float()) < 2e-2


def _block():
    from recant_b200.block import GDNBlock
    G = golden()
    sd = {k: v for k, v in G.items() if k not in ("x", "out", "y")}
    return G, GDNBlock.from_state(sd, HIDDEN, HK, HV)


# The block amplifies rounding differences: re-running the reference's own block with its LoRA
# products as separate ops instead of one addmm moves the output by 3 % (relative Frobenius), so
# end-to-end comparisons use 5e-2; the stages above are compared tightly.
BLOCK_TOL = 5e-2


def test_block_forward_matches_reference_output():
    G, blk = _block()
    with torch.no_grad():
        out = blk(G["x"].to(torch.bfloat16).cuda())
    torch.cuda.synchronize()
    assert rel(out.float(), G["out"]) < BLOCK_TOL, rel(out.float(), G["out"])


def test_block_out_proj_input_and_out_proj_pinned_separately():
    """The end-to-end 5e-2 above, split at out_proj's NVFP4 re-quantization: (1) out_proj's input y
    (the gated norm's output, before it is quantized) against the reference's own y (captured by a
    forward pre-hook on the reference's out_proj, tests/golden/make_golden.py) at the bf16 GDN bound
    2e-2; (2) this library's out_proj applied to the reference's y against the reference's output,
    at 1e-4 (the same NVFP4 codes, fp32 accumulation: measured 3.4e-5)."""
    G, blk = _block()
    seen = {}
    hook = blk.out_proj.register_forward_pre_hook(lambda mod, args: seen.setdefault("y", args[0].detach().clone()))
    try:
        with torch.no_grad():
            blk(G["x"].to(torch.bfloat16).cuda())
    finally:
        hook.remove()
    torch.cuda.synchronize()
    assert rel(seen["y"].float(), G["y"]) < 2e-2, rel(seen["y"].float(), G["y"])
    with torch.no_grad():
        out = blk.out_proj(G["y"].to(torch.bfloat16).cuda())
    torch.cuda.synchronize()
    assert rel(out.float(), G["out"]) < 1e-4, rel(out.float(), G["out"])


def test_block_backward_matches_oracle():
    G, blk = _block()
    blk.set_stochastic_backward(False)   # the oracle quantizes dy round-to-nearest
    P = oracle_params(G, requires_grad=True)
    x = G["x"].to(torch.bfloat16)
    gen = torch.Generator().manual_seed(9)
    dy = torch.randn(x.shape, generator=gen).to(torch.bfloat16)
    xr = x.clone().requires_grad_(True)
    OB.block_forward(xr, P, HK, HV).backward(dy)
    xd = x.cuda().requires_grad_(True)
    blk(xd).backward(dy.cuda())
    torch.cuda.synchronize()
    errs = {"dx": rel(xd.grad.float(), xr.grad.float())}
    for name in ("in_proj_qkv", "in_proj_z", "out_proj"):
        lin = getattr(blk, name)
        errs[name + ".A"] = rel(lin.lora_A.grad, P[name]["A"].grad)
        errs[name + ".B"] = rel(lin.lora_B.grad, P[name]["B"].grad)
    # dx goes through the in_proj dgrad GEMMs, which re-quantize dqkv / dz to NVFP4: upstream
    # gradients that differ by ~1e-2 (the LoRA-gradient errors) flip the codes of elements next to a
    # decision point, one e2m1 step each, so dx is compared at 1e-1
    tol = {k: (1e-1 if k == "dx" else BLOCK_TOL) for k in errs}
    bad = {k: v for k, v in errs.items() if not v < tol[k]}
    assert not bad, (bad, errs)


def test_block_backward_split_at_the_in_proj_dgrad(monkeypatch):
    """dx's 1e-1 above, split at the in_proj dgrad GEMMs that re-quantize their upstream gradients:
    (1) the gradients arriving at the four input projections' outputs (qkv, z, b, a) against the
    oracle's at the bf16 bound 2e-2 (measured 4e-3 to 9e-3); (2) this block's backward started from
    the oracle's own upstream gradients against the oracle's dx at 1e-2 (measured 3.3e-3, the bf16
    rounding of dx's four summed contributions). The projections' outputs are taken from the
    module-level functions both forwards call (oracle.block.qlinear; grouped_linear and gdn_gates
    here)."""
    import recant_b200.block as BM
    G, blk = _block()
    blk.set_stochastic_backward(False)   # the oracle quantizes dy round-to-nearest
    P = oracle_params(G, requires_grad=True)
    x = G["x"].to(torch.bfloat16)
    dy = torch.randn(x.shape, generator=torch.Generator().manual_seed(9)).to(torch.bfloat16)
    kept_o = []
    ql = OB.qlinear

    def qlinear_kept(x_, p, grouped=False):
        y = ql(x_, p, grouped)
        y.retain_grad()
        kept_o.append(y)
        return y

    monkeypatch.setattr(OB, "qlinear", qlinear_kept)
    xr = x.clone().requires_grad_(True)
    OB.block_forward(xr, P, HK, HV).backward(dy)
    up_o = dict(zip(("qkv", "z", "b", "a"), (t.grad for t in kept_o[:4])))
    kept = {}
    gl, gg = BM.grouped_linear, BM.gdn_gates

    def grouped_kept(x_, lins, h=None, base=None):
        out = gl(x_, lins, h=h, base=base)
        for t in out:
            t.retain_grad()
        kept["qkv"], kept["z"] = out
        return out

    def gates_kept(a, b, A_log, dt_bias):
        a.retain_grad()
        b.retain_grad()
        kept["a"], kept["b"] = a, b
        return gg(a, b, A_log, dt_bias)

    monkeypatch.setattr(BM, "grouped_linear", grouped_kept)
    monkeypatch.setattr(BM, "gdn_gates", gates_kept)
    xd = x.cuda().requires_grad_(True)
    blk(xd).backward(dy.cuda())
    torch.cuda.synchronize()
    errs = {n: rel(kept[n].grad.float(), up_o[n].float()) for n in up_o}
    assert all(v < 2e-2 for v in errs.values()), errs
    kept.clear()
    xd2 = x.cuda().requires_grad_(True)
    blk(xd2)
    names = ("qkv", "z", "b", "a")
    torch.autograd.backward([kept[n] for n in names],
                            [up_o[n].to(kept[n].dtype).cuda().reshape(kept[n].shape) for n in names])
    torch.cuda.synchronize()
    assert rel(xd2.grad.float(), xr.grad.float()) < 1e-2, rel(xd2.grad.float(), xr.grad.float())


def test_block_stochastic_backward_is_unbiased_around_rn():
    """The default (reference) backward rounds dy stochastically: its input gradient scatters around
    the round-to-nearest one."""
    G, blk = _block()
    x = G["x"].to(torch.bfloat16).cuda()
    dy = torch.randn(x.shape, generator=torch.Generator().manual_seed(2)).to(torch.bfloat16).cuda()
    grads = []
    for sr in (False, True, True):
        blk.set_stochastic_backward(sr)
        xd = x.clone().requires_grad_(True)
        blk(xd).backward(dy)
        grads.append(xd.grad.float())
    assert rel(grads[1], grads[0]) < 0.3 and rel(grads[1], grads[2]) > 0


def test_conv_silu_with_cached_prefix():
    """The decode path's conv: cached prefix prev [B, C, 3] in front of x, the next prefix =
    cat(prev, x)[..., -3:] (layers.py:157-166), and dx with the prefix entering u."""
    from recant_b200.block import conv_silu
    gen = torch.Generator().manual_seed(6)
    for T in (1, 2, 37):
        B, C, s1, s2 = 2, 512, 128, 256
        x = torch.randn(B, T, C, generator=gen).to(torch.bfloat16)
        prev = torch.randn(B, C, 3, generator=gen).to(torch.bfloat16)
        w = (torch.randn(C, 1, 4, generator=gen) * 0.4).to(torch.bfloat16)
        dy = torch.randn(B, T, C, generator=gen).to(torch.bfloat16)
        xr = x.clone().requires_grad_(True)
        cat = torch.cat([prev, xr.transpose(1, 2)], -1)
        ref = F.silu(F.conv1d(cat, w, groups=C)).transpose(1, 2)
        ref.backward(dy)
        xd = x.cuda().requires_grad_(True)
        q, k, v, state = conv_silu(xd, w.cuda(), s1, s2, prev=prev.cuda(), want_state=True)
        out = torch.cat([q, k, v], -1)
        out.backward(dy.cuda())
        torch.cuda.synchronize()
        assert torch.equal(state.cpu(), cat[..., -3:].detach()), T
        assert rel(out.float(), ref.float()) < 1e-2, T
        assert rel(xd.grad.float(), xr.grad.float()) < 1e-2, T


# The cache carries states that no NVFP4 stage follows: compared at the bf16 GDN bound. The outputs pass
# through out_proj, which re-quantizes its input y to NVFP4: on the 2 x 40 prefill y differs from the
# reference by 4.8e-3 (qkv's GEMM summation order, 1e-3, grown by the delta rule), which flips e2m1
# codes and moves the output by 5.8 %, while this out_proj on that same y matches the reference's
# out_proj on it to 9e-6. So the outputs are compared at 1e-1.
STATE_TOL = 2e-2
DECODE_OUT_TOL = 1e-1


def test_block_decode_with_cache_matches_reference():
    """GDNBlock driven as the serving engine drives GatedDeltaNet (serve/engine.py:107-119): a prefill,
    single-token steps and a short chunk through a LayerCache, against the reference block's outputs
    and cache states (tests/golden/block_decode_golden.npz)."""
    from block_util import decode_golden
    from recant_b200 import _lib as L
    from recant_b200.block import LayerCache
    G, blk = _block()
    D = decode_golden()
    x = D["x"].to(torch.bfloat16).cuda()
    cache = LayerCache()
    prof = L.LaunchProfiler(capacity=4096)
    prof.start()
    with torch.no_grad():
        for i, (s, e) in enumerate(D["calls"].tolist()):
            out = blk(x[:, s:e], cache, s)
            torch.cuda.synchronize()
            assert rel(cache.conv_state.float(), D[f"conv_state{i}"]) < STATE_TOL, i
            if f"rec_state{i}" in D:
                assert rel(cache.rec_state, D[f"rec_state{i}"]) < STATE_TOL, i
            assert rel(out.float(), D[f"out{i}"]) < DECODE_OUT_TOL, (i, rel(out.float(), D[f"out{i}"]))
    names = {n for n, _ in prof.read()[0]}
    assert "gdn_recurrent" in names and "block_conv_state" in names, names


def test_block_decode_out_proj_input_and_out_proj_pinned_separately():
    """The decode outputs' 1e-1 above, split at out_proj's NVFP4 re-quantization, call by call: out_proj's
    input y against the reference's (forward pre-hook on the reference's out_proj) at the bf16 GDN bound,
    and this library's out_proj on the reference's y against the reference's output at 1e-4."""
    from block_util import decode_golden
    from recant_b200.block import LayerCache
    G, blk = _block()
    D = decode_golden()
    x = D["x"].to(torch.bfloat16).cuda()
    cache = LayerCache()
    seen = []
    hook = blk.out_proj.register_forward_pre_hook(lambda mod, args: seen.append(args[0].detach().clone()))
    try:
        with torch.no_grad():
            for s, e in D["calls"].tolist():
                blk(x[:, s:e], cache, s)
    finally:
        hook.remove()
    torch.cuda.synchronize()
    assert len(seen) == len(D["calls"])
    for i, y in enumerate(seen):
        assert rel(y.float(), D[f"y{i}"]) < STATE_TOL, (i, rel(y.float(), D[f"y{i}"]))
        with torch.no_grad():
            out = blk.out_proj(D[f"y{i}"].to(torch.bfloat16).cuda())
        torch.cuda.synchronize()
        assert rel(out.float(), D[f"out{i}"]) < 1e-4, (i, rel(out.float(), D[f"out{i}"]))


def test_cache_pieces_equal_one_call():
    """Feeding a sequence in pieces with the carried state gives the one-call result for the stages
    without a per-call scale: the conv exactly, the GDN op (recurrent and chunked pieces) to fp32
    rounding. (The NVFP4 projections quantize each call with its own global scale, as the reference
    does, so the block's outputs depend on how the sequence is cut.)"""
    from oracle import inputs as I
    from recant_b200 import gdn_b200
    from recant_b200.block import conv_silu
    gen = torch.Generator().manual_seed(8)
    x = torch.randn(2, 70, 512, generator=gen).to(torch.bfloat16).cuda()
    w = (torch.randn(512, 1, 4, generator=gen) * 0.4).to(torch.bfloat16).cuda()
    cuts = ((0, 33), (33, 34), (34, 36), (36, 70))
    with torch.no_grad():
        full = torch.cat(conv_silu(x, w, 128, 256), -1)
        prev, parts = None, []
        for s0, e0 in cuts:
            q, k, v, prev = conv_silu(x[:, s0:e0].contiguous(), w, 128, 256, prev=prev, want_state=True)
            parts.append(torch.cat([q, k, v], -1))
        assert torch.equal(torch.cat(parts, 1), full)
        inp = {n: t.cuda() for n, t in I.gdn_inputs(2, 70, 2, 4, 128, dtype=torch.float32, seed=8).items()}
        o_full, h_full = gdn_b200(**inp, output_final_state=True)
        h, outs = None, []
        for s0, e0 in cuts:
            piece = {n: t[:, s0:e0].contiguous() for n, t in inp.items()}
            o, h = gdn_b200(**piece, initial_state=h, output_final_state=True)
            outs.append(o)
    assert rel(torch.cat(outs, 1), o_full) < 1e-4 and rel(h, h_full) < 1e-4


def test_decode_graph_replays_the_eager_decode_step():
    """The CUDA-graph decode step (static cache, updated in place) gives exactly the eager cache path's
    outputs and states, step after step."""
    from recant_b200.block import DecodeGraph, LayerCache
    G, blk = _block()
    gen = torch.Generator().manual_seed(13)
    x = torch.randn(3, 12, HIDDEN, generator=gen).to(torch.bfloat16).cuda()
    with torch.no_grad():
        eager = LayerCache()
        blk(x[:, :6], eager)
        graphed = eager.fork()
        step = DecodeGraph(blk, graphed, B=3)
        for t in range(6, 12):
            ref = blk(x[:, t:t + 1], eager)
            out = step(x[:, t:t + 1])
            assert torch.equal(out, ref), t
        assert torch.equal(graphed.conv_state, eager.conv_state)
        assert torch.equal(graphed.rec_state, eager.rec_state)


def test_block_lora_grads_without_input_grad():
    """With x needing no gradient (config 2 trains LoRA only) the NVFP4 dgrads are skipped, as the
    reference's autograd skips them; the LoRA gradients are those of the full backward."""
    G, blk = _block()
    blk.set_stochastic_backward(False)
    x = G["x"].to(torch.bfloat16).cuda()
    dy = torch.randn(x.shape, generator=torch.Generator().manual_seed(4)).to(torch.bfloat16).cuda()
    grads = []
    for need in (True, False):
        for p in blk.parameters():
            p.grad = None
        xi = x.clone().requires_grad_(need)
        blk(xi).backward(dy)
        grads.append({n: p.grad.clone() for n, p in blk.named_parameters() if p.grad is not None})
    assert grads[0].keys() == grads[1].keys() and len(grads[0]) == 6
    for n in grads[0]:
        assert rel(grads[1][n], grads[0][n]) < 1e-6, n


def test_block_with_fused_lora_epilogue():
    """The opt-in path that adds LoRA inside the NVFP4 GEMM epilogue (rounded as the reference's addmm
    and three-op forms) matches the reference block and gives the addmm path's LoRA gradients."""
    import recant_b200.block as RB
    G, blk = _block()
    blk.set_stochastic_backward(False)
    x = G["x"].to(torch.bfloat16).cuda()
    dy = torch.randn(x.shape, generator=torch.Generator().manual_seed(6)).to(torch.bfloat16).cuda()
    outs, grads = [], []
    old = RB.FUSED_LORA_EPILOGUE
    try:
        for fused in (False, True):
            RB.FUSED_LORA_EPILOGUE = fused
            for p in blk.parameters():
                p.grad = None
            xi = x.clone().requires_grad_(True)
            out = blk(xi)
            out.backward(dy)
            outs.append(out.detach().float())
            grads.append({n: p.grad.clone() for n, p in blk.named_parameters() if p.grad is not None})
    finally:
        RB.FUSED_LORA_EPILOGUE = old
    assert rel(outs[1], G["out"]) < BLOCK_TOL, rel(outs[1], G["out"])
    for n in grads[0]:
        assert rel(grads[1][n], grads[0][n]) < 2e-2, (n, rel(grads[1][n], grads[0][n]))


@pytest.mark.parametrize("rht", [True, False])
def test_gated_rmsnorm_quant_equals_norm_then_quantize(rht):
    """The fused gated norm + NVFP4 quantize (rb2_gated_rmsnorm_nvfp4_fwd) gives bit-identical y, codes,
    scales, blocked scales and global scale to the norm followed by the stand-alone quantizer, and the
    same input gradients."""
    from recant_b200 import block as BL
    from recant_b200 import nvfp4 as N
    gen = torch.Generator().manual_seed(11 + rht)
    M, K = 300, 4096
    x = (torch.randn(M * K // 128, 128, generator=gen) * 2).to(torch.bfloat16).cuda().requires_grad_(True)
    z = torch.randn(M * K // 128, 128, generator=gen).to(torch.bfloat16).cuda().requires_grad_(True)
    w = (1 + 0.1 * torch.randn(128, generator=gen)).cuda()
    y1, a1 = BL.gated_rmsnorm_quant(x, z, w, K, rht)
    x2, z2 = x.detach().clone().requires_grad_(True), z.detach().clone().requires_grad_(True)
    y2 = BL.gated_rmsnorm(x2, z2, w)
    a2 = N.quantize_fast(y2.detach().reshape(M, K), rht, False)
    torch.cuda.synchronize()
    assert torch.equal(y1, y2)
    assert torch.equal(a1.codes, a2.codes) and torch.equal(a1.scales.view(torch.uint8), a2.scales.view(torch.uint8))
    assert torch.equal(a1.blocked, a2.blocked) and torch.equal(a1.gscale, a2.gscale)
    dy = torch.randn(y1.shape, generator=gen).to(torch.bfloat16).cuda()
    y1.backward(dy)
    y2.backward(dy)
    assert torch.equal(x.grad, x2.grad) and torch.equal(z.grad, z2.grad)


def test_block_with_and_without_norm_quant_fusion_agree():
    """A block large enough for the fused norm + quantize path gives the same output and LoRA
    gradients with the fusion switched off (the stand-alone norm and quantizer)."""
    from recant_b200 import block as BL
    gen = torch.Generator(device="cuda").manual_seed(21)
    blk = BL.GDNBlock(512, 2, 4).cuda()
    for lin in blk.projections():
        lin.load_weight(torch.randn(lin.out_features, lin.in_features, device="cuda", generator=gen) * 0.02)
    for lin in (blk.in_proj_qkv, blk.in_proj_z, blk.out_proj):
        lin.add_lora(16, 32, "cuda")
        with torch.no_grad():
            lin.lora_B.normal_(0, 0.01, generator=gen)
    x = torch.randn(2, 600, 512, device="cuda", generator=gen).to(torch.bfloat16)
    dy = torch.randn(2, 600, 512, device="cuda", generator=gen).to(torch.bfloat16)
    outs, grads = [], []
    for fuse in (True, False):
        BL.FUSE_NORM_QUANT = fuse
        try:
            for p in blk.parameters():
                p.grad = None
            for lin in blk.projections():
                lin.stochastic_backward = False
            y = blk(x)
            y.backward(dy)
            outs.append(y.detach())
            grads.append([blk.out_proj.lora_A.grad.clone(), blk.in_proj_qkv.lora_A.grad.clone()])
        finally:
            BL.FUSE_NORM_QUANT = True
    assert torch.equal(outs[0], outs[1])
    for a, b in zip(*grads):
        assert torch.equal(a, b)
