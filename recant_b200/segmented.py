"""Segmented and context-parallel GDN: the affine state hand-off.

Per chunk the state update is affine in the incoming state,
    S_{c+1} = A_c S_c + b_c,   A_c = gamma_c I - k~_c^T W_c,   b_c = k~_c^T U_c,
so a run of chunks (a *segment*) maps S_in to  S_out = M S_in + S0  with  M = A_n ... A_1  and
S0 = S_out(S_in = 0). The backward is the transposed map: dS_in = M^T dS_out + dS0 with dS0 the
initial-state gradient for dS_out = 0.

Forward of one long sequence split into segments (all on the tensor-core path, chunk-aligned
segment boundaries so the chunking equals the unsegmented op's):
  1. per-chunk prep once (rb2_gdn_fwd_ex stage 1, segments passed as cu_seqlens);
  2. state-only walk  -> S0 of every segment (in parallel over segments);
  3. transition walk  -> M of every segment (U = 0, S_0 = I);
  4. prefix over segments (and, with a process group, over ranks via all_gather of the rank's
     composed (M_r, S0_r)) -> the true S_in of every segment; every fold is one launch of the
     fold kernel (rb2_gdn_state_fold);
  5. normal walk from those S_in -> o, per-chunk states, final state.
Backward: state-only reversed walk -> dS0; suffix over segments (and ranks, all_gather of d_r);
normal reversed walk from the true dS_out; chunk backward.

With a process group (context parallelism), each rank passes its contiguous token shard of the
sequence; only rank 0's ``initial_state`` and the last rank's final-state gradient are used.
The collectives per layer are one all_gather of 2 x Hv x 128 x 128 fp32 in the forward and one
of Hv x 128 x 128 fp32 in the backward, plus, only when the final state is requested, its broadcast
from the last rank and the broadcast of its gradient.
"""
from __future__ import annotations

import ctypes as C

import torch

from . import _lib as L
from .gdn import _PATHS, _stream


def state_fold(M, c=None, s0=None, *, transpose=False, identity=False, states=True, mode=None, prefix=None):
    """Fold the affine maps M [n, H, 128, 128] (offsets c, same shape, None = 0) from the start
    value s0 [H, 128, 128] (None = zero, or the identity with ``identity``) on the GPU.
    Forward: x_0 = s0, x_{k+1} = M_k x_k + c_k; transposed: from k = n-1 down, x = M_k^T x + c_k.
    ``mode`` 2: forward order applying M_k^T (pass transposed maps to apply the originals; the
    fastest form). ``prefix`` = (Mp, cp): maps applied first, in the same mode, values not recorded.
    Returns (values entering every map [n, H, 128, 128] or None, value after the last map)."""
    n, H = int(M.shape[0]), int(M.shape[1])
    dev = M.device
    if mode is None:
        mode = 1 if transpose else 0
    Mp, cp = prefix if prefix is not None else (None, None)
    n_p = 0 if Mp is None else int(Mp.shape[0])
    out_states = torch.empty_like(M) if states else None
    out_final = torch.empty(H, 128, 128, dtype=torch.float32, device=dev)
    L.check(L.lib().rb2_gdn_state_fold_ex(L.ptr(M), L.ptr(c), n, L.ptr(Mp if n_p else None), L.ptr(cp if n_p else None),
                                          n_p, L.ptr(s0), H, 128, int(mode), int(identity), L.ptr(out_states),
                                          L.ptr(out_final), _stream(dev)), "gdn_state_fold")
    return out_states, out_final


def _t(M):
    """Maps with their last two dimensions transposed (contiguous): mode-2 folds apply the originals."""
    return M.transpose(-1, -2).contiguous()


class _SegmentedGDN(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, g, beta, initial_state, seg_len, group, scale, want_final):
        if q.shape[0] != 1 or q.dtype != torch.bfloat16:
            raise ValueError("recant_b200.gdn_segmented: needs B == 1 and bfloat16 inputs (tensor-core path)")
        if seg_len % 64:
            raise ValueError("recant_b200.gdn_segmented: segment length must be a multiple of 64")
        _, T, Hk, dk = q.shape
        Hv, dv = v.shape[2], v.shape[3]
        dev = q.device
        q, k, v = (t.contiguous() for t in (q, k, v))
        g = g.to(torch.float32).contiguous()
        beta = beta.to(torch.bfloat16).contiguous()
        bounds = list(range(0, T, seg_len)) + [T]
        cu = torch.tensor(bounds, dtype=torch.int64, device=dev)
        n = len(bounds) - 1
        scale = float(dk ** -0.5 if scale is None else scale)
        lib = L.lib()
        path = _PATHS["fast"]
        saved, scratch = C.c_size_t(0), C.c_size_t(0)
        L.check(lib.rb2_gdn_workspace_split(1, T, n, Hk, Hv, dk, dv, L.BF16, path, C.byref(saved), C.byref(scratch)),
                "gdn_workspace_split")
        wsb = saved.value
        ws = torch.empty(wsb, dtype=torch.uint8, device=dev)
        common = lambda: (L.ptr(q), L.ptr(k), L.ptr(v), L.ptr(g), L.ptr(beta))
        dims = (1, T, n, Hk, Hv, dk, dv, L.BF16, path, scale)
        st = _stream(dev)

        def fwd(h0, o, hT, stages, walk):
            L.check(lib.rb2_gdn_fwd_ex(*common(), L.ptr(h0), L.ptr(cu), *dims, L.ptr(o), L.ptr(hT), L.ptr(ws), wsb,
                                       st, stages, walk), "gdn_fwd_ex")

        S0 = torch.empty(n, Hv, dk, dv, dtype=torch.float32, device=dev)
        Ms = torch.empty(n, Hv, dk, dk, dtype=torch.float32, device=dev)
        fwd(None, None, S0, 1 | 2, 1)     # prep + state-only walk
        fwd(None, None, Ms, 2, 2)         # transition walk
        s0 = torch.zeros(Hv, dk, dv, dtype=torch.float32, device=dev)
        world, rank = 1, 0
        if group is not None:
            import torch.distributed as dist
            world, rank = dist.get_world_size(group), dist.get_rank(group)
        if initial_state is not None and rank == 0:
            s0 = initial_state.reshape(Hv, dk, dv).to(torch.float32)
        M_all = None
        MsT = _t(Ms)
        s0 = s0.contiguous()
        if world > 1:
            import torch.distributed as dist
            packed = torch.empty(2, Hv, dk, dk, dtype=torch.float32, device=dev)
            # the rank's composed map M_r = M_{n-1} ... M_0 and its output c_r for its true input
            # (rank 0: the initial state; others: zero)
            _, packed[0] = state_fold(MsT, identity=True, states=False, mode=2)
            _, packed[1] = state_fold(MsT, S0, s0, states=False, mode=2)
            gathered = torch.empty(world, 2, Hv, dk, dk, dtype=torch.float32, device=dev)
            dist.all_gather_into_tensor(gathered, packed, group=group)
            M_all = gathered[:, 0].contiguous()
            c_all = gathered[:, 1].contiguous()
            # this rank's input: the preceding ranks' maps from zero (rank 0's output already holds
            # the initial state), then its own segments, in one launch
            if rank > 0:
                s0 = torch.zeros_like(s0)
            S_in, _ = state_fold(MsT, S0, s0, mode=2, prefix=(_t(M_all[:rank]), c_all[:rank]) if rank else None)
        else:
            S_in, _ = state_fold(MsT, S0, s0, mode=2)
        o = torch.empty(1, T, Hv, dv, dtype=torch.bfloat16, device=dev)
        hT = torch.empty(n, Hv, dk, dv, dtype=torch.float32, device=dev)
        fwd(S_in, o, hT, 2, 0)            # normal walk from the true segment inputs
        final = hT[n - 1].unsqueeze(0).clone()
        if world > 1 and want_final:  # the whole sequence's final state lives on the last rank
            import torch.distributed as dist
            dist.broadcast(final, src=world - 1, group=group)
        ctx.save_for_backward(q, k, v, g, beta, cu, S_in)
        ctx.ws, ctx.wsb, ctx.scratch_bytes, ctx.Ms, ctx.M_all = ws, wsb, scratch.value, Ms, M_all
        ctx.dims, ctx.n, ctx.group, ctx.world, ctx.rank = dims, n, group, world, rank
        ctx.has_h0 = initial_state is not None
        ctx.want_final = want_final
        ctx.set_materialize_grads(False)
        if not want_final:
            ctx.mark_non_differentiable(final)
        return o, final

    @staticmethod
    def backward(ctx, do, dfinal):
        q, k, v, g, beta, cu, S_in = ctx.saved_tensors
        ws, wsb, Ms, dims, n = ctx.ws, ctx.wsb, ctx.Ms, ctx.dims, ctx.n
        dev = q.device
        lib = L.lib()
        st = _stream(dev)
        if do is None:
            do = torch.zeros(1, q.shape[1], v.shape[2], v.shape[3], dtype=torch.bfloat16, device=dev)
        do = do.to(torch.bfloat16).contiguous()
        _, T, Hv, dv = do.shape
        dk = q.shape[-1]
        common = (L.ptr(q), L.ptr(k), L.ptr(v), L.ptr(g), L.ptr(beta), L.ptr(S_in), L.ptr(cu))
        dq, dkk, dvv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
        dg = torch.empty_like(g)
        dbeta = torch.empty_like(beta)
        dS0 = torch.empty(n, Hv, dk, dv, dtype=torch.float32, device=dev)
        scratch = torch.empty(max(ctx.scratch_bytes, 1), dtype=torch.uint8, device=dev)

        def bwd(dhT, dh0, stages, walk):
            L.check(lib.rb2_gdn_bwd_ex(*common, *dims, L.ptr(do), L.ptr(dhT), L.ptr(dq), L.ptr(dkk), L.ptr(dvv),
                                       L.ptr(dg), L.ptr(dbeta), L.ptr(dh0), L.ptr(ws), wsb, L.ptr(scratch),
                                       ctx.scratch_bytes, st, stages, walk), "gdn_bwd_ex")

        bwd(None, dS0, 1, 1)              # state-only reversed walk: dS_in for dS_out = 0
        # gradient of the whole sequence's final state: the last rank's
        d_last = torch.zeros(Hv, dk, dv, dtype=torch.float32, device=dev)
        if dfinal is not None:
            d_last = dfinal.reshape(Hv, dk, dv).to(torch.float32).clone()
        if ctx.world > 1:
            import torch.distributed as dist
            if ctx.want_final:  # (every rank decides alike: the final state was requested or not)
                dist.broadcast(d_last, src=ctx.world - 1, group=ctx.group)
            # this rank's left-boundary gradient for a zero right-boundary gradient
            _, d = state_fold(Ms, dS0, transpose=True, states=False)
            d_all = torch.empty(ctx.world, Hv, dk, dv, dtype=torch.float32, device=dev)
            dist.all_gather_into_tensor(d_all, d, group=ctx.group)
            # the following ranks' maps (transposed, last rank first), then this rank's segments
            later = ctx.world - 1 - ctx.rank
            pre = (ctx.M_all[ctx.rank + 1:], d_all[ctx.rank + 1:]) if later else None
            dS_out, _ = state_fold(Ms, dS0, d_last, transpose=True, prefix=pre)
        else:
            dS_out, _ = state_fold(Ms, dS0, d_last, transpose=True)
        dh0 = torch.empty(n, Hv, dk, dv, dtype=torch.float32, device=dev)
        bwd(dS_out, dh0, 1, 0)            # normal reversed walk
        bwd(None, None, 2, 0)             # chunk backward
        d_init = dh0[0].unsqueeze(0) if (ctx.has_h0 and ctx.rank == 0) else None
        return dq, dkk, dvv, dg, dbeta, d_init, None, None, None, None


def gdn_segmented(q, k, v, g, beta, initial_state=None, output_final_state=False, *, segment_len=1024,
                  group=None, scale=None):
    """GDN over one long sequence (B == 1) in chunk-aligned segments processed in parallel, with
    the affine hand-off; with ``group`` (a torch.distributed process group) the sequence is
    context-parallel: every rank passes its contiguous shard. Same semantics as ``gdn_b200``."""
    o, final = _SegmentedGDN.apply(q, k, v, g, beta, initial_state, int(segment_len), group, scale,
                                   bool(output_final_state))
    return o, (final if output_final_state else None)
