"""Installs the B200 KDA kernels behind Sophia's own module seams.

Mirrors the reference's runtime-hook pattern
(``ml/training/pretrain/engine/sm120_concurrent_ffn.py:425-430``), which swaps
``SophiaKDA._fla_chunk_kda`` and ``CausalDepthwiseConv1d.forward`` per module:

* ``SophiaKDA._fla_chunk_kda`` / ``_fla_fused_recurrent_kda``
  (``ml/runtime/model/attention.py:296-312``) return this package's
  ``chunk_kda`` / ``fused_recurrent_kda``;
* ``SophiaKDA.forward`` (``attention.py:373-420``) is replaced per instance by
  a version that sends the pre-conv projections straight to ``kda_layer``, so
  the ShortConv+SiLU, L2 norms, gate and beta run fused in the chunk kernels.
  A cached continuation (``start_pos > 0`` with ``use_cache``, the decode
  step) goes to ``kda_decode``: the conv with the module's ``conv_state``
  history and the recurrence from ``recurrent_state`` in one kernel, both
  states updated as the reference updates them.  The replacement keeps the
  reference's pad-mask, cache and output-gate semantics and defers to the
  original forward when a cached continuation needs gradients, when the
  tensors are not on CUDA, or when the module's ``kda_backend`` is
  ``"reference"``.

The reference package is never imported here: modules are recognised by
their class name and attributes.
"""

from __future__ import annotations

from types import MethodType

import torch

from .ops import HEAD_DIM, chunk_kda, fused_recurrent_kda, gated_rms_norm, kda_decode, kda_layer

PAD_LOGIT = -1.0e4  # attention.py:17


def _is_kda(m) -> bool:
    return type(m).__name__ == "SophiaKDA" and hasattr(m, "q_conv") and hasattr(m, "_run_kda")


def _gate_out(self, x: torch.Tensor, output: torch.Tensor) -> torch.Tensor:
    bsz, seqlen, _ = x.shape
    gate_logits = (self.output_gate(x) if self.output_gate_full_rank
                   else self.output_gate_up(self.output_gate_down(x)))
    # output RMSNorm and sigmoid gate in one kernel (attention.py:416-419)
    output = gated_rms_norm(output.to(dtype=x.dtype), gate_logits.view(bsz, seqlen, self.num_heads, self.head_dim),
                            self.output_norm.weight, float(self.output_norm.eps))
    return self.o_proj(output.reshape(bsz, seqlen, self.inner_dim))


def _cached_step(self, x: torch.Tensor) -> torch.Tensor:
    """start_pos > 0 with the cache: no pad mask (attention.py:377-380), conv
    history from conv_state, initial state from recurrent_state, both
    rewritten after the step (attention.py:244-257,398-410)."""
    bsz, seqlen, _ = x.shape
    H, D = self.num_heads, self.head_dim
    self.ensure_batch_capacity(int(bsz))
    qp, kp, vp = self.q_proj(x), self.k_proj(x), self.v_proj(x)
    decay_logits = self.decay_up(self.decay_down(x)).view(bsz, seqlen, H, D)
    beta_logits = self.beta_proj(x)
    with torch.no_grad():
        output, final_state = kda_decode(
            qp.view(bsz, seqlen, H, D), kp.view(bsz, seqlen, H, D), vp.view(bsz, seqlen, H, D),
            decay_logits, beta_logits, self.A_log, self.dt_bias, self.q_conv.weight, self.k_conv.weight,
            self.v_conv.weight, self.conv_state[:bsz], lower_bound=self.lower_bound,
            initial_state=self.recurrent_state[:bsz])
        self.recurrent_state[:bsz].copy_(final_state)
    return _gate_out(self, x, output)


def _fused_forward(self, x: torch.Tensor, *, start_pos: int = 0) -> torch.Tensor:
    if not x.is_cuda or self.backend == "reference" or self.conv_kernel != 4 or self.head_dim != HEAD_DIM:
        return self._b200_reference_forward(x, start_pos=start_pos)
    if int(start_pos) > 0 and self.use_cache:
        if torch.is_grad_enabled() and (x.requires_grad or any(p.requires_grad for p in self.parameters())):
            return self._b200_reference_forward(x, start_pos=start_pos)
        return _cached_step(self, x)
    bsz, seqlen, _ = x.shape
    H, D, inner = self.num_heads, self.head_dim, self.inner_dim
    if self.use_cache:
        self.ensure_batch_capacity(int(bsz))
    pad_mask = getattr(self, "_pad_mask", None) if int(start_pos) == 0 else None
    if pad_mask is not None:
        keep = pad_mask[:, :seqlen].to(dtype=x.dtype).unsqueeze(-1)
        x = x * keep
    qp, kp, vp = self.q_proj(x), self.k_proj(x), self.v_proj(x)
    decay_logits = self.decay_up(self.decay_down(x)).view(bsz, seqlen, H, D)
    beta_logits = self.beta_proj(x)
    if pad_mask is not None:
        drop = ~pad_mask[:, :seqlen].bool()
        decay_logits = decay_logits.masked_fill(drop[:, :, None, None], PAD_LOGIT)
        beta_logits = beta_logits.masked_fill(drop[:, :, None], PAD_LOGIT)
    output, final_state = kda_layer(
        qp.view(bsz, seqlen, H, D), kp.view(bsz, seqlen, H, D), vp.view(bsz, seqlen, H, D),
        decay_logits, beta_logits, self.A_log, self.dt_bias,
        self.q_conv.weight, self.k_conv.weight, self.v_conv.weight,
        lower_bound=self.lower_bound, output_final_state=bool(self.use_cache))
    if self.use_cache:
        with torch.no_grad():
            self.recurrent_state[:bsz].copy_(final_state.detach().to(torch.float32))
            hist = self.conv_kernel - 1
            for index, proj in enumerate((qp, kp, vp)):
                seq = torch.cat((proj.new_zeros(bsz, hist, inner), proj), dim=1)[:, -hist:]
                self.conv_state[:bsz, index].copy_(seq.transpose(1, 2).detach().to(torch.float32))
    return _gate_out(self, x, output)


def install(model: torch.nn.Module, *, fuse_conv: bool = True) -> dict[str, object]:
    """Patches every ``SophiaKDA`` in ``model``; returns a small report."""
    patched = 0
    for module in model.modules():
        if not _is_kda(module):
            continue
        module._fla_chunk_kda = lambda: chunk_kda
        module._fla_fused_recurrent_kda = lambda: fused_recurrent_kda
        if fuse_conv and not hasattr(module, "_b200_reference_forward"):
            module._b200_reference_forward = module.forward
            module.forward = MethodType(_fused_forward, module)
        patched += 1
    from . import _lib
    lib = _lib.load()
    return {"kda_modules": patched, "library": str(_lib.LIB_PATH),
            "version": lib.kda_b200_version().decode(), "fused_conv": bool(fuse_conv)}
