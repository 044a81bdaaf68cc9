"""Host-side operators of the B200 KDA layer.

``chunk_kda`` mirrors flash-linear-attention's ``chunk_kda`` (the callee of
Sophia's ``SophiaKDA._fla_chunk_kda`` seam, ``ml/runtime/model/attention.py:
305-312,349-365``; contract ``fla/ops/kda/chunk.py:167-411``): same argument
names and meaning, same ``ValueError``/``AssertionError`` checks, same
``(o, final_state)`` result.  ``kda_layer`` adds the ShortConv(+SiLU) of
``CausalDepthwiseConv1d`` (``attention.py:32-60``) in front, fused into the
chunk prologue.  Both dispatch to ``libkda_b200.so`` through its C ABI; there
is no other implementation behind them.

Precision follows the inputs, as in flash-linear-attention: bf16 (or fp16)
q/k/v run the bf16 tensor-core kernels with an fp32 state; float32 q/k/v run
the fp32 kernels (fp32 arithmetic throughout, the precision of the
reference's own ``_reference_kda``).

Every kernel call is a ``torch.library.custom_op`` (namespace ``sophia_b200``)
with a fake implementation and a registered autograd formula, so a model that
is ``torch.compile``d -- Sophia compiles its training model,
``ml/training/pretrain/engine/sm120_graph_runner.py:71-75`` -- traces these
ops as opaque nodes instead of into the ctypes calls (the reference's own hook
reaches the same end with ``torch.compiler.disable``,
``ml/training/pretrain/engine/sm120_concurrent_ffn.py:425``).  Inside the ops
autocast is off: inputs are used at the dtype they arrive in, as
flash-linear-attention's ``autocast_custom_fwd``/``bwd`` keep them
(``fla/ops/kda/chunk.py:25,119``).
"""

from __future__ import annotations

from typing import Optional

import torch
from torch import Tensor

from . import _lib

__all__ = ["chunk_kda", "kda_layer", "kda_decode", "fused_recurrent_kda", "gated_rms_norm"]

HEAD_DIM = 128


def _ptr(t: Tensor | None) -> int | None:
    return None if t is None or t.numel() == 0 else t.data_ptr()


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _fp32_mode(q: Tensor, k: Tensor, v: Tensor) -> bool:
    return torch.float32 in (q.dtype, k.dtype, v.dtype)


def _num_seqs(q: Tensor, cu_seqlens: Tensor | None) -> int:
    return q.shape[0] if cu_seqlens is None else cu_seqlens.shape[0] - 1


def _saved_bytes(fp32: bool, tokens: int, H: int, N: int, packed: bool) -> int:
    lib = _lib.load()
    if fp32:
        return int(lib.kda_b200_f32_saved_bytes(tokens, H, N))
    return int(lib.kda_b200_saved_bytes(tokens, H, N, int(packed)))


def _empty(like: Tensor, dtype=torch.float32) -> Tensor:
    return like.new_empty((0,), dtype=dtype)


# --------------------------------------------------------------------------- layer


def _kda_fwd_impl(q, k, v, g, beta, A_log, dt_bias, conv_q, conv_k, conv_v, h0, cu_seqlens, scale, lower_bound,
                  output_final_state, training):
    """Returns (o in the compute dtype, final state or empty, saved buffer or empty)."""
    with torch.autocast("cuda", enabled=False):
        lib = _lib.load()
        fp32 = _fp32_mode(q, k, v)
        cdt = torch.float32 if fp32 else torch.bfloat16
        B, T, H, D = q.shape
        N = _num_seqs(q, cu_seqlens)
        qb, kb, vb, gb, bb = (x.to(cdt).contiguous() for x in (q, k, v, g, beta))
        A = A_log.float().contiguous()
        dtb = dt_bias.float().contiguous()
        convs = [None if c is None else c.float().contiguous() for c in (conv_q, conv_k, conv_v)]
        h0c = None if h0 is None else h0.float().contiguous()
        cu = None if cu_seqlens is None else cu_seqlens.to(torch.int32).contiguous()
        packed = cu is not None
        o = torch.empty(B, T, H, D, device=q.device, dtype=cdt)
        ht = (torch.empty(N, H, D, D, device=q.device, dtype=torch.float32) if output_final_state
              else _empty(q))
        saved = (torch.empty(_saved_bytes(fp32, B * T, H, N, packed), device=q.device, dtype=torch.uint8)
                 if training else _empty(q, torch.uint8))
        if fp32:
            ws_bytes, fn = lib.kda_b200_f32_fwd_workspace_bytes(B * T, H, N, int(training)), lib.kda_b200_fwd_f32
        else:
            ws_bytes, fn = lib.kda_b200_fwd_workspace_bytes(B * T, H, N, int(packed), int(training)), lib.kda_b200_fwd
        ws = torch.empty(ws_bytes, device=q.device, dtype=torch.uint8)
        _lib.check(fn(
            _ptr(qb), _ptr(kb), _ptr(vb), _ptr(gb), _ptr(bb), _ptr(A), _ptr(dtb),
            _ptr(convs[0]), _ptr(convs[1]), _ptr(convs[2]), _ptr(h0c), _ptr(cu),
            B, T, H, D, N, float(scale), float(lower_bound),
            _ptr(o), _ptr(ht), _ptr(saved), saved.numel(), _ptr(ws), ws.numel(), _stream()))
        return o, ht, saved


@torch.library.custom_op("sophia_b200::kda_fwd", mutates_args=(), device_types="cuda")
def _kda_fwd(q: Tensor, k: Tensor, v: Tensor, g: Tensor, beta: Tensor, A_log: Tensor, dt_bias: Tensor,
             conv_q: Optional[Tensor], conv_k: Optional[Tensor], conv_v: Optional[Tensor],
             h0: Optional[Tensor], cu_seqlens: Optional[Tensor], scale: float, lower_bound: float,
             output_final_state: bool, training: bool) -> tuple[Tensor, Tensor, Tensor]:
    return _kda_fwd_impl(q, k, v, g, beta, A_log, dt_bias, conv_q, conv_k, conv_v, h0, cu_seqlens, scale,
                         lower_bound, output_final_state, training)


@_kda_fwd.register_fake
def _(q, k, v, g, beta, A_log, dt_bias, conv_q, conv_k, conv_v, h0, cu_seqlens, scale, lower_bound,
      output_final_state, training):
    fp32 = _fp32_mode(q, k, v)
    B, T, H, D = q.shape
    N = _num_seqs(q, cu_seqlens)
    o = q.new_empty((B, T, H, D), dtype=torch.float32 if fp32 else torch.bfloat16)
    ht = q.new_empty((N, H, D, D) if output_final_state else (0,), dtype=torch.float32)
    nbytes = _saved_bytes(fp32, int(B * T), int(H), int(N), cu_seqlens is not None) if training else 0
    return o, ht, q.new_empty((nbytes,), dtype=torch.uint8)


def _kda_bwd_impl(q, k, v, g, beta, A_log, dt_bias, conv_q, conv_k, conv_v, h0, cu_seqlens, saved, do, dht, scale,
                  lower_bound, want_dh0):
    """Returns (dq, dk, dv, dg, dbeta, dA_log, ddt_bias, dconv_q, dconv_k, dconv_v, dh0); absent ones empty."""
    with torch.autocast("cuda", enabled=False):
        lib = _lib.load()
        fp32 = _fp32_mode(q, k, v)
        cdt = torch.float32 if fp32 else torch.bfloat16
        B, T, H, D = q.shape
        N = _num_seqs(q, cu_seqlens)
        qb, kb, vb, gb, bb = (x.to(cdt).contiguous() for x in (q, k, v, g, beta))
        A = A_log.float().contiguous()
        dtb = dt_bias.float().contiguous()
        convs = [None if c is None else c.float().contiguous() for c in (conv_q, conv_k, conv_v)]
        conv = convs[0] is not None
        cu = None if cu_seqlens is None else cu_seqlens.to(torch.int32).contiguous()
        dob = do.to(cdt).contiguous()
        dhtc = None if dht is None else dht.float().contiguous()
        dq, dk, dv, dg = (torch.empty_like(qb) for _ in range(4))
        dbeta = torch.empty_like(bb)
        dA = torch.empty_like(A)
        ddt = torch.empty_like(dtb)
        dconvs = [torch.empty_like(c) if conv else _empty(q) for c in convs]
        dh0 = torch.empty(N, H, D, D, device=q.device, dtype=torch.float32) if want_dh0 else _empty(q)
        if fp32:
            ws_bytes, fn = lib.kda_b200_f32_bwd_workspace_bytes(B * T, H, N), lib.kda_b200_bwd_f32
        else:
            ws_bytes, fn = lib.kda_b200_bwd_workspace_bytes(B * T, H, N, int(cu is not None)), lib.kda_b200_bwd
        ws = torch.empty(ws_bytes, device=q.device, dtype=torch.uint8)
        h0c = None if h0 is None else h0.float().contiguous()
        _lib.check(fn(
            _ptr(qb), _ptr(kb), _ptr(vb), _ptr(gb), _ptr(bb), _ptr(A), _ptr(dtb),
            _ptr(convs[0]), _ptr(convs[1]), _ptr(convs[2]), _ptr(h0c), _ptr(cu),
            B, T, H, D, N, float(scale), float(lower_bound), _ptr(saved), saved.numel(),
            _ptr(dob), _ptr(dhtc), _ptr(dq), _ptr(dk), _ptr(dv), _ptr(dg), _ptr(dbeta),
            _ptr(dA), _ptr(ddt), _ptr(dconvs[0]), _ptr(dconvs[1]), _ptr(dconvs[2]), _ptr(dh0),
            _ptr(ws), ws.numel(), _stream()))
        return dq, dk, dv, dg, dbeta, dA, ddt, dconvs[0], dconvs[1], dconvs[2], dh0


@torch.library.custom_op("sophia_b200::kda_bwd", mutates_args=(), device_types="cuda")
def _kda_bwd(q: Tensor, k: Tensor, v: Tensor, g: Tensor, beta: Tensor, A_log: Tensor, dt_bias: Tensor,
             conv_q: Optional[Tensor], conv_k: Optional[Tensor], conv_v: Optional[Tensor],
             h0: Optional[Tensor], cu_seqlens: Optional[Tensor], saved: Tensor, do: Tensor,
             dht: Optional[Tensor], scale: float, lower_bound: float, want_dh0: bool
             ) -> tuple[Tensor, Tensor, Tensor, Tensor, Tensor, Tensor, Tensor, Tensor, Tensor, Tensor, Tensor]:
    return _kda_bwd_impl(q, k, v, g, beta, A_log, dt_bias, conv_q, conv_k, conv_v, h0, cu_seqlens, saved, do, dht,
                         scale, lower_bound, want_dh0)


@_kda_bwd.register_fake
def _(q, k, v, g, beta, A_log, dt_bias, conv_q, conv_k, conv_v, h0, cu_seqlens, saved, do, dht, scale,
      lower_bound, want_dh0):
    cdt = torch.float32 if _fp32_mode(q, k, v) else torch.bfloat16
    B, T, H, D = q.shape
    N = _num_seqs(q, cu_seqlens)
    act = [q.new_empty(x.shape, dtype=cdt) for x in (q, k, v, g, beta)]
    dA = A_log.new_empty(A_log.shape, dtype=torch.float32)
    ddt = dt_bias.new_empty(dt_bias.shape, dtype=torch.float32)
    dconvs = [q.new_empty(c.shape if c is not None else (0,), dtype=torch.float32) for c in (conv_q, conv_k, conv_v)]
    dh0 = q.new_empty((N, H, D, D) if want_dh0 else (0,), dtype=torch.float32)
    return (*act, dA, ddt, *dconvs, dh0)


def _kda_setup_context(ctx, inputs, output):
    (q, k, v, g, beta, A_log, dt_bias, conv_q, conv_k, conv_v, h0, cu_seqlens, scale, lower_bound,
     _ofs, training) = inputs
    if not training:
        raise RuntimeError("kda_fwd was called with training=False but autograd needs its backward")
    ctx.save_for_backward(q, k, v, g, beta, A_log, dt_bias, conv_q, conv_k, conv_v, h0, cu_seqlens, output[2])
    ctx.scale, ctx.lower_bound = scale, lower_bound


def _kda_grads(ctx, do, dht, bwd):
    q, k, v, g, beta, A_log, dt_bias, conv_q, conv_k, conv_v, h0, cu, saved = ctx.saved_tensors
    dht = None if dht is None or dht.numel() == 0 else dht
    if do is None:
        do = torch.zeros(q.shape, device=q.device, dtype=torch.float32 if _fp32_mode(q, k, v) else torch.bfloat16)
    grads = bwd(q, k, v, g, beta, A_log, dt_bias, conv_q, conv_k, conv_v, h0, cu, saved, do, dht,
                ctx.scale, ctx.lower_bound, h0 is not None)
    dq, dk, dv, dg, dbeta, dA, ddt, dcq, dck, dcv, dh0 = grads
    cast = lambda d, x: None if x is None else d.to(x.dtype)  # noqa: E731
    return (cast(dq, q), cast(dk, k), cast(dv, v), cast(dg, g), cast(dbeta, beta), cast(dA, A_log),
            cast(ddt, dt_bias), None if conv_q is None else dcq.to(conv_q.dtype),
            None if conv_k is None else dck.to(conv_k.dtype), None if conv_v is None else dcv.to(conv_v.dtype),
            None if h0 is None else dh0.to(h0.dtype), None, None, None, None, None)


def _kda_backward(ctx, do, dht, _dsaved):
    return _kda_grads(ctx, do, dht, _kda_bwd)


_kda_fwd.register_autograd(_kda_backward, setup_context=_kda_setup_context)


class _KdaEager(torch.autograd.Function):
    """The eager path: the same implementation as the ``sophia_b200::kda_fwd``
    / ``kda_bwd`` custom ops without the custom-op dispatch, and with the saved
    buffer held by the autograd context instead of returned."""

    @staticmethod
    def forward(ctx, q, k, v, g, beta, A_log, dt_bias, conv_q, conv_k, conv_v, h0, cu_seqlens, scale, lower_bound,
                output_final_state):
        training = any(ctx.needs_input_grad)
        o, ht, saved = _kda_fwd_impl(q, k, v, g, beta, A_log, dt_bias, conv_q, conv_k, conv_v, h0, cu_seqlens,
                                     scale, lower_bound, output_final_state, training)
        if training:
            ctx.save_for_backward(q, k, v, g, beta, A_log, dt_bias, conv_q, conv_k, conv_v, h0, cu_seqlens, saved)
            ctx.scale, ctx.lower_bound = scale, lower_bound
        ctx.set_materialize_grads(False)
        return o, ht

    @staticmethod
    def backward(ctx, do, dht):
        return _kda_grads(ctx, do, dht, _kda_bwd_impl)[:15]


def _needs_grad(*tensors) -> bool:
    return torch.is_grad_enabled() and any(t is not None and t.requires_grad for t in tensors)


def _layer(q, k, v, g, beta, A_log, dt_bias, conv_q, conv_k, conv_v, h0, cu_seqlens, scale, lower_bound,
           output_final_state):
    if torch.compiler.is_compiling():  # traced: the custom op, an opaque node with a fake
        training = _needs_grad(q, k, v, g, beta, A_log, dt_bias, conv_q, conv_k, conv_v, h0)
        o, ht, _ = _kda_fwd(q, k, v, g, beta, A_log, dt_bias, conv_q, conv_k, conv_v, h0, cu_seqlens, float(scale),
                            float(lower_bound), bool(output_final_state), training)
    else:
        o, ht = _KdaEager.apply(q, k, v, g, beta, A_log, dt_bias, conv_q, conv_k, conv_v, h0, cu_seqlens,
                                float(scale), float(lower_bound), bool(output_final_state))
    return o.to(q.dtype), (ht if output_final_state else None)


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
    for name, x in (("q", q), ("k", k), ("v", v)):
        if x.dtype not in (torch.float32, torch.bfloat16, torch.float16):
            raise NotImplementedError(f"{name} must be float32, bfloat16 or float16, got {x.dtype}")
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
    chunk size 64, K = V = 128, H == HV.  float32 q/k/v select the fp32
    kernels; bf16/fp16 the bf16 kernels.
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
    return _layer(q, k, v, g, beta, A_log, dt_bias, None, None, None, initial_state, cu_seqlens, scale,
                  lower_bound, output_final_state)


def kda_layer(q, k, v, g, beta, A_log, dt_bias, conv_q, conv_k, conv_v, *, lower_bound=-5.0,
              scale=None, initial_state=None, output_final_state=False, cu_seqlens=None):
    """ShortConv(k=4)+SiLU on q/k/v followed by the KDA recurrence, fused.

    q, k, v: pre-conv projections ``[B, T, H, 128]``; conv_*: ``[H*128, 4]``
    depthwise taps (``CausalDepthwiseConv1d.weight``); the conv history starts
    at zero for every sequence (``attention.py:40-45``).  Returns
    ``(o, final_state | None)``; gradients reach every input.  float32 q/k/v
    select the fp32 kernels.
    """
    for c in (conv_q, conv_k, conv_v):
        if c is None or tuple(c.shape) != (q.shape[2] * HEAD_DIM, 4):
            raise ValueError("conv taps must be [H*128, 4] tensors")
    _check_common(q, k, v, g, beta, initial_state, cu_seqlens, lower_bound)
    if scale is None:
        scale = q.shape[-1] ** -0.5
    return _layer(q, k, v, g, beta, A_log, dt_bias, conv_q, conv_k, conv_v, initial_state, cu_seqlens, scale,
                  lower_bound, output_final_state)


# --------------------------------------------------------------------------- decode


def _kda_recurrent_impl(q, k, v, g, beta, A_log, dt_bias, h0, cu_seqlens, scale, lower_bound, output_final_state):
    with torch.autocast("cuda", enabled=False):
        fp32 = q.dtype == torch.float32
        dt = torch.float32 if fp32 else torch.bfloat16
        B, T, H, _ = q.shape
        xs = [x.to(dt).contiguous() for x in (q, k, v, g, beta)]
        o = torch.empty(B, T, H, HEAD_DIM, device=q.device, dtype=dt)
        N = _num_seqs(q, cu_seqlens)
        ht = (torch.empty(N, H, HEAD_DIM, HEAD_DIM, device=q.device, dtype=torch.float32) if output_final_state
              else _empty(q))
        cu = None if cu_seqlens is None else cu_seqlens.to(torch.int32).contiguous()
        h0c = None if h0 is None else h0.float().contiguous()
        A_log32, dt_bias32 = A_log.float().contiguous(), dt_bias.float().contiguous()
        _lib.check(_lib.load().kda_b200_recurrent(
            *(_ptr(x) for x in xs), _ptr(A_log32), _ptr(dt_bias32), _ptr(h0c), _ptr(cu),
            B, T, H, HEAD_DIM, N, int(fp32), float(scale), float(lower_bound), _ptr(o), _ptr(ht), _stream()))
        return o, ht


@torch.library.custom_op("sophia_b200::kda_recurrent", mutates_args=(), device_types="cuda")
def _kda_recurrent(q: Tensor, k: Tensor, v: Tensor, g: Tensor, beta: Tensor, A_log: Tensor, dt_bias: Tensor,
                   h0: Optional[Tensor], cu_seqlens: Optional[Tensor], scale: float, lower_bound: float,
                   output_final_state: bool) -> tuple[Tensor, Tensor]:
    return _kda_recurrent_impl(q, k, v, g, beta, A_log, dt_bias, h0, cu_seqlens, scale, lower_bound,
                               output_final_state)


@_kda_recurrent.register_fake
def _(q, k, v, g, beta, A_log, dt_bias, h0, cu_seqlens, scale, lower_bound, output_final_state):
    B, T, H, _ = q.shape
    N = _num_seqs(q, cu_seqlens)
    o = q.new_empty((B, T, H, HEAD_DIM), dtype=torch.float32 if q.dtype == torch.float32 else torch.bfloat16)
    return o, q.new_empty((N, H, HEAD_DIM, HEAD_DIM) if output_final_state else (0,), dtype=torch.float32)


def _kda_decode_impl(q, k, v, g, beta, A_log, dt_bias, conv_q, conv_k, conv_v, conv_state, h0, scale, lower_bound):
    with torch.autocast("cuda", enabled=False):
        if conv_state.dtype != torch.float32 or not conv_state.is_contiguous():
            raise ValueError("conv_state must be a contiguous float32 tensor [B, 3, H*128, 3]")
        fp32 = q.dtype == torch.float32
        dt = torch.float32 if fp32 else torch.bfloat16
        B, T, H, _ = q.shape
        xs = [x.to(dt).contiguous() for x in (q, k, v, g, beta)]
        taps = [c.float().contiguous() for c in (conv_q, conv_k, conv_v)]
        o = torch.empty(B, T, H, HEAD_DIM, device=q.device, dtype=dt)
        ht = torch.empty(B, H, HEAD_DIM, HEAD_DIM, device=q.device, dtype=torch.float32)
        h0c = None if h0 is None else h0.float().contiguous()
        A_log32, dt_bias32 = A_log.float().contiguous(), dt_bias.float().contiguous()
        _lib.check(_lib.load().kda_b200_decode(
            *(_ptr(x) for x in xs), _ptr(A_log32), _ptr(dt_bias32), *(_ptr(c) for c in taps), _ptr(conv_state),
            _ptr(h0c), None, B, T, H, HEAD_DIM, B, int(fp32), float(scale), float(lower_bound), _ptr(o), _ptr(ht),
            _stream()))
        return o, ht


@torch.library.custom_op("sophia_b200::kda_decode", mutates_args=("conv_state",), device_types="cuda")
def _kda_decode(q: Tensor, k: Tensor, v: Tensor, g: Tensor, beta: Tensor, A_log: Tensor, dt_bias: Tensor,
                conv_q: Tensor, conv_k: Tensor, conv_v: Tensor, conv_state: Tensor, h0: Optional[Tensor],
                scale: float, lower_bound: float) -> tuple[Tensor, Tensor]:
    return _kda_decode_impl(q, k, v, g, beta, A_log, dt_bias, conv_q, conv_k, conv_v, conv_state, h0, scale,
                            lower_bound)


@_kda_decode.register_fake
def _(q, k, v, g, beta, A_log, dt_bias, conv_q, conv_k, conv_v, conv_state, h0, scale, lower_bound):
    B, T, H, _ = q.shape
    o = q.new_empty((B, T, H, HEAD_DIM), dtype=torch.float32 if q.dtype == torch.float32 else torch.bfloat16)
    return o, q.new_empty((B, H, HEAD_DIM, HEAD_DIM), dtype=torch.float32)


def kda_decode(q, k, v, g, beta, A_log, dt_bias, conv_q, conv_k, conv_v, conv_state, *, lower_bound=-5.0,
               scale=None, initial_state=None):
    """Cached continuation of ``SophiaKDA.forward`` (``start_pos > 0``): the
    ShortConv with its history (``_short_convolution``, ``attention.py:226-258``)
    and the token-by-token recurrence from ``initial_state`` (``_run_kda``'s
    decode, ``:330-348``) in one kernel.  q, k, v: pre-conv projections
    ``[B, T, H, 128]``; conv_state: the module's ``[B, 3, H*128, 3]`` fp32
    history, updated in place.  Inference only (no gradients).  Returns
    ``(o, final_state)``."""
    _check_common(q, k, v, g, beta, initial_state, None, lower_bound)
    if _needs_grad(q, k, v, g, beta, A_log, dt_bias, conv_q, conv_k, conv_v, initial_state):
        raise NotImplementedError("kda_decode has no backward; use kda_layer / chunk_kda for training")
    if scale is None:
        scale = q.shape[-1] ** -0.5
    fn = _kda_decode if torch.compiler.is_compiling() else _kda_decode_impl
    o, ht = fn(q, k, v, g, beta, A_log, dt_bias, conv_q, conv_k, conv_v, conv_state, initial_state, float(scale),
               float(lower_bound))
    return o.to(v.dtype), ht


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
    if _needs_grad(q, k, v, g, beta, A_log, dt_bias, initial_state):
        return chunk_kda(q, k, v, g, beta, scale=scale, initial_state=initial_state,
                         output_final_state=output_final_state, use_qk_l2norm_in_kernel=True,
                         use_gate_in_kernel=True, use_beta_sigmoid_in_kernel=True, cu_seqlens=cu_seqlens,
                         safe_gate=True, lower_bound=lower_bound, A_log=A_log, dt_bias=dt_bias)
    if scale is None:
        scale = q.shape[-1] ** -0.5
    fn = _kda_recurrent if torch.compiler.is_compiling() else _kda_recurrent_impl
    o, ht = fn(q, k, v, g, beta, A_log, dt_bias, initial_state, cu_seqlens, float(scale), float(lower_bound),
               bool(output_final_state))
    return o.to(v.dtype), (ht if output_final_state else None)


# --------------------------------------------------------------------------- gated output norm


def _gn_io(o: Tensor, g: Tensor) -> torch.dtype:
    return torch.float32 if torch.float32 in (o.dtype, g.dtype) else torch.bfloat16


def _gated_norm_fwd_impl(o, g, weight, eps):
    with torch.autocast("cuda", enabled=False):
        io = _gn_io(o, g)
        oc, gc = o.to(io).contiguous(), g.to(io).contiguous()
        w = weight.float().contiguous()
        rows = oc.numel() // HEAD_DIM
        y = torch.empty_like(oc)
        _lib.check(_lib.load().kda_b200_gated_norm_fwd(_ptr(oc), _ptr(gc), _ptr(w), rows, HEAD_DIM, float(eps),
                                                       int(io == torch.float32), _ptr(y), _stream()))
        return y


@torch.library.custom_op("sophia_b200::gated_norm_fwd", mutates_args=(), device_types="cuda")
def _gated_norm_fwd(o: Tensor, g: Tensor, weight: Tensor, eps: float) -> Tensor:
    return _gated_norm_fwd_impl(o, g, weight, eps)


@_gated_norm_fwd.register_fake
def _(o, g, weight, eps):
    return o.new_empty(o.shape, dtype=_gn_io(o, g))


def _gated_norm_bwd_impl(dy, o, g, weight, eps):
    with torch.autocast("cuda", enabled=False):
        io = _gn_io(o, g)
        oc, gc = o.to(io).contiguous(), g.to(io).contiguous()
        w = weight.float().contiguous()
        rows = oc.numel() // HEAD_DIM
        dyc = dy.to(io).contiguous()
        d_o, d_g = torch.empty_like(oc), torch.empty_like(gc)
        dw = torch.empty(HEAD_DIM, device=oc.device, dtype=torch.float32)
        lib = _lib.load()
        ws = torch.empty(max(16, lib.kda_b200_gated_norm_workspace_bytes(rows, HEAD_DIM)), device=oc.device,
                         dtype=torch.uint8)
        _lib.check(lib.kda_b200_gated_norm_bwd(_ptr(dyc), _ptr(oc), _ptr(gc), _ptr(w), rows, HEAD_DIM, float(eps),
                                               int(io == torch.float32), _ptr(d_o), _ptr(d_g), _ptr(dw),
                                               _ptr(ws), ws.numel(), _stream()))
        return d_o, d_g, dw


@torch.library.custom_op("sophia_b200::gated_norm_bwd", mutates_args=(), device_types="cuda")
def _gated_norm_bwd(dy: Tensor, o: Tensor, g: Tensor, weight: Tensor, eps: float) -> tuple[Tensor, Tensor, Tensor]:
    return _gated_norm_bwd_impl(dy, o, g, weight, eps)


@_gated_norm_bwd.register_fake
def _(dy, o, g, weight, eps):
    io = _gn_io(o, g)
    return o.new_empty(o.shape, dtype=io), g.new_empty(g.shape, dtype=io), weight.new_empty((HEAD_DIM,),
                                                                                           dtype=torch.float32)


def _gn_setup_context(ctx, inputs, output):
    o, g, weight, eps = inputs
    ctx.save_for_backward(o, g, weight)
    ctx.eps = eps


def _gn_grads(ctx, dy, bwd):
    o, g, weight = ctx.saved_tensors
    d_o, d_g, dw = bwd(dy, o, g, weight, ctx.eps)
    return d_o.to(o.dtype), d_g.to(g.dtype), dw.to(weight.dtype), None


def _gn_backward(ctx, dy):
    return _gn_grads(ctx, dy, _gated_norm_bwd)


_gated_norm_fwd.register_autograd(_gn_backward, setup_context=_gn_setup_context)


class _GnEager(torch.autograd.Function):
    """Eager path of the gated norm: the custom ops' implementation without their dispatch."""

    @staticmethod
    def forward(ctx, o, g, weight, eps):
        ctx.save_for_backward(o, g, weight)
        ctx.eps = eps
        return _gated_norm_fwd_impl(o, g, weight, eps)

    @staticmethod
    def backward(ctx, dy):
        return _gn_grads(ctx, dy, _gated_norm_bwd_impl)


def gated_rms_norm(o: Tensor, g: Tensor, weight: Tensor, eps: float = 1e-5) -> Tensor:
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
    fn = _gated_norm_fwd if torch.compiler.is_compiling() else _GnEager.apply
    return fn(o, g, weight, float(eps)).to(torch.promote_types(o.dtype, g.dtype))
