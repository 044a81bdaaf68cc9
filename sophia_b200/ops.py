"""Host-side operators of the B200 KDA layer.

``chunk_kda`` mirrors flash-linear-attention's ``chunk_kda`` (the callee of
Sophia's ``SophiaKDA._fla_chunk_kda`` seam, ``ml/runtime/model/attention.py:
305-312,349-365``; contract ``fla/ops/kda/chunk.py:167-411``): same argument
names and meaning, same ``ValueError``/``AssertionError`` checks, same
``(o, final_state)`` result.  ``kda_layer`` adds the ShortConv(+SiLU) of
``CausalDepthwiseConv1d`` (``attention.py:32-60``) in front, fused into the
chunk prologue.  Both dispatch to ``libkda_b200.so`` through its C ABI; there
is no other implementation behind them.
"""

from __future__ import annotations

import torch

from . import _lib

__all__ = ["chunk_kda", "kda_layer", "fused_recurrent_kda", "gated_rms_norm"]

HEAD_DIM = 128


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _prep(x: torch.Tensor) -> torch.Tensor:
    return x.to(torch.bfloat16).contiguous()


class _KdaFunction(torch.autograd.Function):
    """q/k/v [B,T,H,128] (pre-conv when conv taps are given), g [B,T,H,128] gate
    logits, beta [B,T,H] beta logits; everything differentiable."""

    @staticmethod
    def forward(ctx, q, k, v, g, beta, A_log, dt_bias, conv_q, conv_k, conv_v, h0, cu_seqlens,
                scale, lower_bound, output_final_state):
        lib = _lib.load()
        out_dtype = q.dtype
        B, T, H, D = q.shape
        N = B if cu_seqlens is None else cu_seqlens.numel() - 1
        qb, kb, vb, gb, bb = (_prep(x) for x in (q, k, v, g, beta))
        A = A_log.float().contiguous()
        dtb = dt_bias.float().contiguous()
        convs = [None if c is None else c.float().contiguous() for c in (conv_q, conv_k, conv_v)]
        h0c = None if h0 is None else h0.float().contiguous()
        cu = None if cu_seqlens is None else cu_seqlens.to(torch.int32).contiguous()
        training = any(ctx.needs_input_grad)
        packed = int(cu is not None)
        o = torch.empty_like(qb)
        ht = torch.empty(N, H, D, D, device=q.device, dtype=torch.float32) if output_final_state else None
        saved = None
        if training:
            saved = torch.empty(lib.kda_b200_saved_bytes(B * T, H, N, packed), device=q.device, dtype=torch.uint8)
        ws = torch.empty(lib.kda_b200_fwd_workspace_bytes(B * T, H, N, packed, int(training)),
                         device=q.device, dtype=torch.uint8)
        _lib.check(lib.kda_b200_fwd(
            _ptr(qb), _ptr(kb), _ptr(vb), _ptr(gb), _ptr(bb), _ptr(A), _ptr(dtb),
            _ptr(convs[0]), _ptr(convs[1]), _ptr(convs[2]), _ptr(h0c), _ptr(cu),
            B, T, H, D, N, float(scale), float(lower_bound),
            _ptr(o), _ptr(ht), _ptr(saved), 0 if saved is None else saved.numel(),
            _ptr(ws), ws.numel(), _stream()))
        ctx.save_for_backward(qb, kb, vb, gb, bb, A, dtb, *convs, h0c, cu, saved)
        ctx.meta = (B, T, H, D, N, float(scale), float(lower_bound), out_dtype,
                    q.dtype, k.dtype, v.dtype, g.dtype, beta.dtype, h0 is not None)
        return o.to(out_dtype), ht

    @staticmethod
    def backward(ctx, do, dht):
        lib = _lib.load()
        qb, kb, vb, gb, bb, A, dtb, cq, ck, cv, h0c, cu, saved = ctx.saved_tensors
        (B, T, H, D, N, scale, lower_bound, out_dtype, qd, kd, vd, gd, bd, has_h0) = ctx.meta
        conv = cq is not None
        dob = _prep(do)
        dhtc = None if dht is None else dht.float().contiguous()
        dq, dk, dv, dg = (torch.empty_like(qb) for _ in range(4))
        dbeta = torch.empty_like(bb)
        dA = torch.empty_like(A)
        ddt = torch.empty_like(dtb)
        dcq = torch.empty_like(cq) if conv else None
        dck = torch.empty_like(ck) if conv else None
        dcv = torch.empty_like(cv) if conv else None
        dh0 = torch.empty(N, H, D, D, device=qb.device, dtype=torch.float32) if has_h0 else None
        ws = torch.empty(lib.kda_b200_bwd_workspace_bytes(B * T, H, N, int(cu is not None)),
                         device=qb.device, dtype=torch.uint8)
        _lib.check(lib.kda_b200_bwd(
            _ptr(qb), _ptr(kb), _ptr(vb), _ptr(gb), _ptr(bb), _ptr(A), _ptr(dtb),
            _ptr(cq), _ptr(ck), _ptr(cv), _ptr(h0c), _ptr(cu),
            B, T, H, D, N, scale, lower_bound, _ptr(saved), saved.numel(),
            _ptr(dob), _ptr(dhtc), _ptr(dq), _ptr(dk), _ptr(dv), _ptr(dg), _ptr(dbeta),
            _ptr(dA), _ptr(ddt), _ptr(dcq), _ptr(dck), _ptr(dcv), _ptr(dh0),
            _ptr(ws), ws.numel(), _stream()))
        return (dq.to(qd), dk.to(kd), dv.to(vd), dg.to(gd), dbeta.to(bd), dA, ddt,
                dcq, dck, dcv, dh0, None, None, None, None)


def _check_common(q, k, v, g, beta, initial_state, cu_seqlens, lower_bound):
    if q.device.type != "cuda":
        raise RuntimeError("the B200 KDA kernels require CUDA tensors")
    if q.shape != k.shape:
        raise AssertionError(f"q and k must have the same shape, got q={q.shape} vs k={k.shape}")
    B, T, H, K = q.shape
    if v.shape[2] != H:
        raise NotImplementedError("grouped value heads (HV > H) are not supported")
    if K != HEAD_DIM or v.shape[-1] != HEAD_DIM:
        raise NotImplementedError(f"head dim must be {HEAD_DIM}, got K={K}, V={v.shape[-1]}")
    if tuple(g.shape) != (B, T, H, K):
        raise AssertionError(f"g must have shape [B, T, HV, K]={[B, T, H, K]}, got {list(g.shape)}")
    if tuple(beta.shape) != (B, T, H):
        raise AssertionError(f"beta must have shape [B, T, HV]={[B, T, H]}, got {list(beta.shape)}")
    if cu_seqlens is not None:
        if B != 1:
            raise ValueError(
                f"The batch size is expected to be 1 rather than {B} when using `cu_seqlens`."
                f"Please flatten variable-length inputs before processing.")
        if initial_state is not None and initial_state.shape[0] != len(cu_seqlens) - 1:
            raise ValueError(
                "The number of initial states is expected to be equal to the number of input sequences, "
                f"i.e., {len(cu_seqlens) - 1} rather than {initial_state.shape[0]}.")
    if initial_state is not None:
        assert initial_state.dtype == torch.float32, "initial_state must be in float32."
    if lower_bound is None or not (-5 <= lower_bound < 0):
        raise ValueError(f"`lower_bound` must be in the safe range [-5, 0), got {lower_bound}.")


def chunk_kda(q, k, v, g, beta, scale=None, initial_state=None, output_final_state=False,
              use_qk_l2norm_in_kernel=False, use_gate_in_kernel=False, use_beta_sigmoid_in_kernel=False,
              cu_seqlens=None, cu_seqlens_cpu=None, safe_gate=False, lower_bound=None,
              disable_recompute=False, return_intermediate_states=False, cp_context=None,
              transpose_state_layout=False, **kwargs):
    """Drop-in for ``fla.ops.kda.chunk_kda`` in the configuration Sophia uses.

    q, k, v: ``[B, T, H, 128]`` (post-conv, pre-norm); g: raw gate logits
    ``[B, T, H, 128]``; beta: raw logits ``[B, T, H]``; ``A_log [H]`` and
    ``dt_bias [H*128]`` via keywords.  Returns ``(o, final_state | None)``.
    Supported: ``use_qk_l2norm_in_kernel``, ``use_gate_in_kernel`` and
    ``use_beta_sigmoid_in_kernel`` all true with ``safe_gate=True`` and
    ``-5 <= lower_bound < 0`` (Sophia's call, ``attention.py:349-365``),
    chunk size 64, K = V = 128, H == HV.
    """
    if cp_context is not None:
        raise NotImplementedError("context-parallel KDA is not part of this path")
    if return_intermediate_states or transpose_state_layout:
        raise NotImplementedError("return_intermediate_states / transpose_state_layout are not supported")
    if use_gate_in_kernel:
        assert "A_log" in kwargs, "A_log must be provided when use_gate_in_kernel=True."
    chunk_size = kwargs.pop("chunk_size", 64)
    if chunk_size not in (32, 64):
        raise ValueError(f"`chunk_size` must be either 32 or 64 for KDA, got {chunk_size}.")
    if chunk_size != 64:
        raise NotImplementedError("the B200 kernels use 64-token chunks")
    if safe_gate and use_gate_in_kernel and lower_bound is None:
        raise ValueError("`lower_bound` must be specified when `safe_gate=True` and `use_gate_in_kernel=True`.")
    if not (use_qk_l2norm_in_kernel and use_gate_in_kernel and use_beta_sigmoid_in_kernel and safe_gate):
        raise NotImplementedError(
            "the B200 kernels implement the fused configuration: use_qk_l2norm_in_kernel, "
            "use_gate_in_kernel, use_beta_sigmoid_in_kernel and safe_gate all True")
    _check_common(q, k, v, g, beta, initial_state, cu_seqlens, lower_bound)
    A_log, dt_bias = kwargs["A_log"], kwargs.get("dt_bias")
    if dt_bias is None:
        dt_bias = torch.zeros(q.shape[2] * HEAD_DIM, device=q.device, dtype=torch.float32)
    if scale is None:
        scale = q.shape[-1] ** -0.5
    return _KdaFunction.apply(q, k, v, g, beta, A_log, dt_bias, None, None, None, initial_state,
                              cu_seqlens, scale, lower_bound, output_final_state)


def kda_layer(q, k, v, g, beta, A_log, dt_bias, conv_q, conv_k, conv_v, *, lower_bound=-5.0,
              scale=None, initial_state=None, output_final_state=False, cu_seqlens=None):
    """ShortConv(k=4)+SiLU on q/k/v followed by the KDA recurrence, fused.

    q, k, v: pre-conv projections ``[B, T, H, 128]``; conv_*: ``[H*128, 4]``
    depthwise taps (``CausalDepthwiseConv1d.weight``); the conv history starts
    at zero for every sequence (``attention.py:40-45``).  Returns
    ``(o, final_state | None)``; gradients reach every input.
    """
    for c in (conv_q, conv_k, conv_v):
        if c is None or tuple(c.shape) != (q.shape[2] * HEAD_DIM, 4):
            raise ValueError("conv taps must be [H*128, 4] tensors")
    _check_common(q, k, v, g, beta, initial_state, cu_seqlens, lower_bound)
    if scale is None:
        scale = q.shape[-1] ** -0.5
    return _KdaFunction.apply(q, k, v, g, beta, A_log, dt_bias, conv_q, conv_k, conv_v, initial_state,
                              cu_seqlens, scale, lower_bound, output_final_state)


def fused_recurrent_kda(q, k, v, g, beta, A_log=None, dt_bias=None, scale=None, initial_state=None,
                        output_final_state=False, use_qk_l2norm_in_kernel=False, use_gate_in_kernel=False,
                        use_beta_sigmoid_in_kernel=False, lower_bound=None, cu_seqlens=None, **kwargs):
    """Decode-step seam (``attention.py:330-348``, flash-linear-attention's
    ``fused_recurrent_kda``): the token-by-token recurrence in fp32 on the GPU
    (``kda_b200_recurrent``), the same configuration as ``chunk_kda``.

    Without gradients (decode) this runs the recurrent kernel; when autograd
    needs gradients of the inputs it evaluates the same recurrence through the
    chunked kernels, which have a backward.  Returns ``(o, final_state | None)``.
    """
    if not (use_qk_l2norm_in_kernel and use_gate_in_kernel and use_beta_sigmoid_in_kernel):
        raise NotImplementedError(
            "the B200 kernels implement the fused configuration: use_qk_l2norm_in_kernel, "
            "use_gate_in_kernel and use_beta_sigmoid_in_kernel all True")
    if A_log is None:
        raise AssertionError("A_log must be provided when use_gate_in_kernel=True.")
    _check_common(q, k, v, g, beta, initial_state, cu_seqlens, lower_bound)
    if dt_bias is None:
        dt_bias = torch.zeros(q.shape[2] * HEAD_DIM, device=q.device, dtype=torch.float32)
    tensors = (q, k, v, g, beta, A_log, dt_bias, initial_state)
    if torch.is_grad_enabled() and any(t is not None and t.requires_grad for t in tensors):
        return chunk_kda(q, k, v, g, beta, scale=scale, initial_state=initial_state,
                         output_final_state=output_final_state, use_qk_l2norm_in_kernel=True,
                         use_gate_in_kernel=True, use_beta_sigmoid_in_kernel=True, cu_seqlens=cu_seqlens,
                         safe_gate=True, lower_bound=lower_bound, A_log=A_log, dt_bias=dt_bias)
    if scale is None:
        scale = q.shape[-1] ** -0.5
    fp32 = q.dtype == torch.float32
    dt = torch.float32 if fp32 else torch.bfloat16
    B, T, H, _ = q.shape
    xs = [x.to(dt).contiguous() for x in (q, k, v, g, beta)]
    o = torch.empty(B, T, H, HEAD_DIM, device=q.device, dtype=dt)
    N = B if cu_seqlens is None else cu_seqlens.numel() - 1
    ht = torch.empty(N, H, HEAD_DIM, HEAD_DIM, device=q.device, dtype=torch.float32) if output_final_state else None
    cu = None if cu_seqlens is None else cu_seqlens.to(torch.int32).contiguous()
    h0 = None if initial_state is None else initial_state.contiguous()
    A_log32, dt_bias32 = A_log.float().contiguous(), dt_bias.float().contiguous()
    _lib.check(_lib.load().kda_b200_recurrent(
        *(_ptr(x) for x in xs), _ptr(A_log32), _ptr(dt_bias32), _ptr(h0), _ptr(cu),
        B, T, H, HEAD_DIM, N, int(fp32), float(scale), float(lower_bound), _ptr(o), _ptr(ht), _stream()))
    return o.to(v.dtype), ht


class _GatedNormFunction(torch.autograd.Function):
    """y = rms_norm(o) * weight * sigmoid(g) over the last dim (128)."""

    @staticmethod
    def forward(ctx, o, g, weight, eps):
        io = torch.float32 if torch.float32 in (o.dtype, g.dtype) else torch.bfloat16
        oc, gc = o.to(io).contiguous(), g.to(io).contiguous()
        w = weight.float().contiguous()
        rows = oc.numel() // HEAD_DIM
        y = torch.empty_like(oc)
        lib = _lib.load()
        _lib.check(lib.kda_b200_gated_norm_fwd(_ptr(oc), _ptr(gc), _ptr(w), rows, HEAD_DIM, float(eps),
                                               int(io == torch.float32), _ptr(y), _stream()))
        ctx.save_for_backward(oc, gc, w)
        ctx.eps = float(eps)
        ctx.dtypes = (o.dtype, g.dtype, weight.dtype)
        return y.to(torch.promote_types(o.dtype, g.dtype))

    @staticmethod
    def backward(ctx, dy):
        oc, gc, w = ctx.saved_tensors
        rows = oc.numel() // HEAD_DIM
        dyc = dy.to(oc.dtype).contiguous()
        d_o, d_g = torch.empty_like(oc), torch.empty_like(gc)
        dw = torch.empty(HEAD_DIM, device=oc.device, dtype=torch.float32)
        lib = _lib.load()
        ws = torch.empty(max(16, lib.kda_b200_gated_norm_workspace_bytes(rows, HEAD_DIM)), device=oc.device,
                         dtype=torch.uint8)
        _lib.check(lib.kda_b200_gated_norm_bwd(_ptr(dyc), _ptr(oc), _ptr(gc), _ptr(w), rows, HEAD_DIM, ctx.eps,
                                               int(oc.dtype == torch.float32), _ptr(d_o), _ptr(d_g), _ptr(dw),
                                               _ptr(ws), ws.numel(), _stream()))
        od, gd, wd = ctx.dtypes
        return d_o.to(od), d_g.to(gd), dw.to(wd), None


def gated_rms_norm(o: torch.Tensor, g: torch.Tensor, weight: torch.Tensor, eps: float = 1e-5) -> torch.Tensor:
    """``rms_norm(o) * weight * sigmoid(g)`` per row of 128 channels: the output
    norm and gate of ``SophiaKDA.forward`` (``ml/runtime/model/attention.py:
    416-419`` with ``RMSNorm``, ``ml/runtime/model/ops.py:49-64``), fused into one
    kernel forward and one backward.  o, g: [..., 128] CUDA tensors of the
    same shape (bf16 or fp32); weight: [128].  Differentiable in o, g, weight.
    """
    if o.shape != g.shape or o.shape[-1] != HEAD_DIM or weight.shape != (HEAD_DIM,):
        raise ValueError(f"gated_rms_norm expects o, g [..., {HEAD_DIM}] of one shape and weight [{HEAD_DIM}], "
                         f"got {tuple(o.shape)}, {tuple(g.shape)}, {tuple(weight.shape)}")
    if not (o.is_cuda and g.is_cuda and weight.is_cuda):
        raise RuntimeError("gated_rms_norm runs on the CUDA kernels only: o, g and weight must be CUDA tensors")
    return _GatedNormFunction.apply(o, g, weight, eps)
