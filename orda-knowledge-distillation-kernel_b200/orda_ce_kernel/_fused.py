"""Autograd wrapper around ``orda_distill_fwdbwd`` (the fused sm_100a kernels).

Semantics follow the reference autograd Functions: the forward computes the losses AND the
gradients (``ops/tied_teacher.py:366-519``), the backward only rescales the stored gradients by
``grad_output * mean_scale`` and casts them to the input dtypes (``ops/tied_teacher.py:529-564``).
Gradient presence matches the reference per mode:

* tied: student hidden, weight, and teacher hidden (all-zero when ``teacher_ce_weight == 0``,
  ``tied_teacher.py:478-479``);
* separate: teacher hidden / weight gradients only when ``teacher_ce_weight > 0``
  (``SeparateFullCEFunction``), otherwise ``None`` (``separate_teacher.py:706-740``);
* precomputed: never any teacher gradient.
"""
from __future__ import annotations

import contextlib
import threading
from dataclasses import dataclass

import ctypes

import torch
from torch.autograd.function import once_differentiable

from . import _native
from ._runtime import default_compute_dtype

_DTYPE_CODE = {torch.float32: _native.F32, torch.float16: _native.F16, torch.bfloat16: _native.BF16}
_DIV_CODE = {"forward": _native.DIV_FORWARD, "reverse": _native.DIV_REVERSE, "jsd": _native.DIV_JSD}
_MODE_CODE = {
    "tied": _native.TEACHER_TIED,
    "separate": _native.TEACHER_SEPARATE,
    "precomputed_logits": _native.TEACHER_LOGITS,
    "precomputed_hidden": _native.TEACHER_HIDDEN,
}


_HOOKS = threading.local()


@contextlib.contextmanager
def instrument(phase_events=None, dweight_done_event=None, dweight_first=False, reserve_sms=0, peer_exchange=None):
    """Attach CUDA events to the fused calls made inside the block (benchmarks / overlap):
    ``phase_events`` - 2*PHASES ``torch.cuda.Event(enable_timing=True)`` recorded around each phase;
    ``dweight_done_event`` - recorded when the weight gradients are complete;
    ``dweight_first`` - run the dW GEMMs before the dH GEMMs;
    ``reserve_sms`` - with ``dweight_first``, SMs the dH GEMMs leave free for a concurrent all-reduce;
    ``peer_exchange`` - a :class:`orda_ce_kernel.parallel.PeerGradientExchange`: the lm_head gradient
    is summed over the data-parallel ranks through peer memory (the returned gradient is the
    exchange's buffer, complete once the current stream reaches it)."""
    prev = getattr(_HOOKS, "value", None)
    _HOOKS.value = (phase_events, dweight_done_event, dweight_first, reserve_sms, peer_exchange)
    try:
        yield
    finally:
        _HOOKS.value = prev


@dataclass(frozen=True)
class FusedSpec:
    mode: str                   # key of _MODE_CODE
    student_ce_weight: float
    teacher_ce_weight: float    # resolved
    kl_weight: float
    kl_temperature: float
    ignore_index: int
    reduction: str
    divergence: str = "forward"
    jsd_beta: float = 0.5
    chunk_rows: int = 0         # 0: library default
    fp32_grad_weight: bool = False
    validate_labels: bool = False


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _operand(t: torch.Tensor, dtype: torch.dtype, pad_cols: int) -> torch.Tensor:
    """Row-major copy-on-need in `dtype`, columns padded with zeros to `pad_cols`, 16-byte aligned base."""
    if t.dtype != dtype:
        t = t.to(dtype)
    if pad_cols != t.shape[1]:
        t = torch.nn.functional.pad(t, (0, pad_cols - t.shape[1]))
    if t.stride(1) != 1 or t.stride(0) != t.shape[1] or t.data_ptr() % 16 != 0:
        t = t.contiguous()
        if t.data_ptr() % 16 != 0:
            t = t.clone()
    return t


def _round8(x: int) -> int:
    return (x + 7) // 8 * 8


def _check_labels(labels: torch.Tensor, vocab: int, ignore_index: int) -> None:
    # same host-side check as the reference ops (ops/tied_teacher.py:630-636)
    valid = (labels == ignore_index) | ((labels >= 0) & (labels < vocab))
    if not bool(valid.all()):
        bad = labels[~valid].tolist()[:5]
        raise ValueError(
            f"labels contains values outside [0, {vocab}) and not equal to ignore_index={ignore_index}: {bad}"
        )


class Prepared:
    """Arguments of one library call plus the tensors that must outlive it."""

    __slots__ = ("args", "keep", "g_hs", "g_ht", "g_w", "g_wt", "out", "status", "h", "h_t", "dev")


def need_grad_flags(student_hidden, teacher_hidden, weight, teacher_weight, spec: FusedSpec) -> list[bool]:
    """Which of (student hidden, teacher hidden, lm_head, teacher lm_head) receive gradients: the
    tensors that require them and, for the teacher, only where a teacher CE term reaches them (tied
    teacher always; separate teacher with a teacher CE weight)."""
    tied, sep = spec.mode == "tied", spec.mode == "separate"
    need_hs = bool(student_hidden.requires_grad)
    need_w = bool(weight.requires_grad)
    need_ht = bool(teacher_hidden is not None and teacher_hidden.requires_grad
                   and (tied or (sep and spec.teacher_ce_weight > 0)))
    need_wt = bool(sep and spec.teacher_ce_weight > 0 and teacher_weight is not None and teacher_weight.requires_grad)
    return [need_hs, need_ht, need_w, need_wt]


def prepare_call(student_hidden, teacher_hidden, weight, teacher_weight, labels, teacher_logits, spec: FusedSpec,
                 vocab_offset: int = 0, vocab_total: int | None = None, need: list[bool] | None = None) -> Prepared:
    """Operands in the compute dtype (the reference's rule), TMA-friendly layout, output buffers and
    the filled ``orda_distill_args_t``. ``weight`` (and a separate teacher's weight) may be a vocab
    shard starting at ``vocab_offset`` of a ``vocab_total``-row lm_head. ``need`` overrides the
    gradient flags (hs, ht, w, wt) that are otherwise read from ``requires_grad``."""
    mode = spec.mode
    dev = student_hidden.device
    if dev.type != "cuda":
        raise RuntimeError("the fused distillation kernels need CUDA tensors (there is no CPU fallback)")
    kl_on = spec.kl_weight != 0.0
    tied, sep = mode == "tied", mode == "separate"
    t_logits_mode, t_hidden_mode = mode == "precomputed_logits", mode == "precomputed_hidden"

    # ---- compute dtype, as each reference Function picks it
    if tied:
        cdt = default_compute_dtype(weight, student_hidden, teacher_hidden)
    elif sep:
        cdt = default_compute_dtype(weight, teacher_weight, student_hidden, teacher_hidden)
    elif t_logits_mode:
        cdt = default_compute_dtype(weight, student_hidden, teacher_logits) if kl_on else default_compute_dtype(weight, student_hidden)
    else:
        cdt = default_compute_dtype(weight, student_hidden, teacher_hidden) if kl_on else default_compute_dtype(weight, student_hidden)
    if cdt not in _DTYPE_CODE:
        cdt = torch.float32

    need_hs, need_ht, need_w, need_wt = (
        need if need is not None else need_grad_flags(student_hidden, teacher_hidden, weight, teacher_weight, spec))

    n, h = student_hidden.shape
    vocab = weight.shape[0]
    is16 = cdt != torch.float32
    hp = _round8(h) if is16 else h
    hs_c = _operand(student_hidden.detach(), cdt, hp)
    w_c = _operand(weight.detach(), cdt, hp)
    ht_c = wt_c = tl_c = None
    h_t = h
    if tied:
        ht_c = _operand(teacher_hidden.detach(), cdt, hp)
        h_t = h
    elif sep or t_hidden_mode:
        h_t = teacher_hidden.shape[1]
        htp = _round8(h_t) if is16 else h_t
        ht_c = _operand(teacher_hidden.detach(), cdt, htp)
        wt_c = _operand(teacher_weight.detach(), cdt, htp)
    elif t_logits_mode:
        tl_c = teacher_logits.detach()
        if tl_c.dtype not in _DTYPE_CODE:
            tl_c = tl_c.float()
        if tl_c.stride(1) != 1:
            tl_c = tl_c.contiguous()
    h_tp = ht_c.shape[1] if ht_c is not None else hp
    labels_c = labels.contiguous()
    if spec.validate_labels:
        _check_labels(labels_c, vocab if vocab_total is None else int(vocab_total), spec.ignore_index)

    f32_acc = spec.fp32_grad_weight or not is16
    wdt = torch.float32 if f32_acc else cdt
    g_hs = torch.empty((n, hp), dtype=cdt, device=dev) if need_hs else None
    g_w = torch.empty((vocab, hp), dtype=wdt, device=dev) if need_w else None
    g_ht = torch.empty((n, h_tp), dtype=cdt, device=dev) if need_ht else None
    g_wt = torch.empty((vocab, h_tp), dtype=wdt, device=dev) if need_wt else None
    out = torch.empty(_native.OUT_SLOTS, dtype=torch.float32, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)

    a = _native.DistillArgs()
    a.abi_version = _native.ABI_VERSION
    a.teacher_mode = _MODE_CODE[mode]
    a.compute_dtype = _DTYPE_CODE[cdt]
    a.teacher_logits_dtype = _DTYPE_CODE[tl_c.dtype] if tl_c is not None else _native.F32
    a.n_rows, a.hidden, a.teacher_hidden, a.vocab = n, hp, h_tp, vocab
    a.vocab_offset = int(vocab_offset)
    a.vocab_total = int(vocab if vocab_total is None else vocab_total)
    a.student_hidden, a.ld_student_hidden = _ptr(hs_c), hs_c.stride(0)
    a.weight, a.ld_weight = _ptr(w_c), w_c.stride(0)
    if ht_c is not None:
        a.teacher_hidden_ptr, a.ld_teacher_hidden = _ptr(ht_c), ht_c.stride(0)
    if wt_c is not None:
        a.teacher_weight, a.ld_teacher_weight = _ptr(wt_c), wt_c.stride(0)
    if tl_c is not None:
        a.teacher_logits, a.ld_teacher_logits = _ptr(tl_c), tl_c.stride(0)
    a.labels = _ptr(labels_c)
    a.student_ce_weight = float(spec.student_ce_weight)
    a.teacher_ce_weight = float(spec.teacher_ce_weight)
    a.kl_weight = float(spec.kl_weight)
    a.kl_temperature = float(spec.kl_temperature)
    a.jsd_beta = float(spec.jsd_beta)
    a.divergence = _DIV_CODE[spec.divergence]
    a.ignore_index = int(spec.ignore_index)
    a.reduction = _native.REDUCTION_MEAN if spec.reduction == "mean" else _native.REDUCTION_SUM
    a.validate_labels = 0
    a.need_grad_student_hidden, a.need_grad_weight = int(need_hs), int(need_w)
    a.need_grad_teacher_hidden, a.need_grad_teacher_weight = int(need_ht), int(need_wt)
    a.chunk_rows = int(spec.chunk_rows)
    a.out_reduced = _ptr(out)
    a.out_row_losses = None
    a.grad_student_hidden, a.grad_weight = _ptr(g_hs), _ptr(g_w)
    a.grad_teacher_hidden, a.grad_teacher_weight = _ptr(g_ht), _ptr(g_wt)
    a.grad_weight_fp32 = int(f32_acc)
    a.device_status = _ptr(status)
    a.grads_include_mean_scale = 1  # dlogits carry 1/count: backward only multiplies by grad_output

    pr = Prepared()
    pr.args, pr.keep = a, (hs_c, w_c, ht_c, wt_c, tl_c, labels_c)
    pr.g_hs, pr.g_ht, pr.g_w, pr.g_wt = g_hs, g_ht, g_w, g_wt
    pr.out, pr.status, pr.h, pr.h_t, pr.dev = out, status, h, h_t, dev
    return pr


def rescale_saved_grads(ctx, grads, grad_output):
    """Backward of the fused Functions: the stored gradients already include the mean scale, so each
    is multiplied by ``grad_output`` - in place on the device (a no-op when grad_output == 1, the
    usual ``loss.backward()``), or out of place where the stored buffer is padded or in another dtype.
    Repeated backward calls (retain_graph) divide out the factor already applied."""
    lib = _native.load()
    go = grad_output.detach().to(torch.float32).reshape(()).contiguous()
    if not hasattr(ctx, "applied"):
        ctx.applied = [None] * len(grads)
    stream = torch.cuda.current_stream(go.device).cuda_stream
    out = []
    for i, (g, cols, dtype) in enumerate(grads):
        if g is None:
            out.append(None)
            continue
        if ctx.applied[i] is not None:
            out.append((g[:, :cols] * (go / ctx.applied[i])).to(dtype))
        elif g.shape[1] == cols and g.dtype == dtype and g.is_contiguous():
            _native.check(lib.orda_scale_grad(g.data_ptr(), g.numel(), _DTYPE_CODE[g.dtype], go.data_ptr(), stream),
                          "orda_scale_grad")
            ctx.applied[i] = go.clone()
            out.append(g)
        else:
            out.append((g[:, :cols] * go).to(dtype))
    return out


def launch_prepared(pr: Prepared, spec: FusedSpec, keep_alive=None) -> None:
    """One ``orda_distill_fwdbwd`` call on the current stream with a workspace from the caching
    allocator; instrumentation hooks of :func:`instrument` are attached here."""
    lib = _native.load()
    a, dev, status = pr.args, pr.dev, pr.status
    hooks = getattr(_HOOKS, "value", None)
    exchange = None
    if hooks is not None:
        ev, done, first, reserve, exchange = hooks
        if ev is not None:
            handles = (ctypes.c_void_p * (2 * _native.PHASES))(*[e.cuda_event for e in ev])
            if keep_alive is not None:
                keep_alive._phase_handles = handles  # the array must outlive the call
            a.phase_events = ctypes.cast(handles, ctypes.c_void_p)
        if done is not None:
            a.dweight_done_event = done.cuda_event
        a.dweight_first = int(bool(first))
        a.overlap_reserve_sms = int(reserve)

    ws_bytes = int(lib.orda_distill_workspace_bytes(a))
    ws = torch.empty(max(ws_bytes, 256), dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    if exchange is not None and pr.g_w is not None:
        exchange.prepare(pr)
        _native.check(lib.orda_distill_fwdbwd_peer(a, ws.data_ptr(), ws_bytes, ctypes.byref(exchange.desc), stream),
                      "orda_distill_fwdbwd_peer")
        exchange.complete()
    else:
        _native.check(lib.orda_distill_fwdbwd(a, ws.data_ptr(), ws_bytes, stream), "orda_distill_fwdbwd")

    if spec.validate_labels:
        code = int(status.item())
        if code != _native.OK:
            raise RuntimeError(f"orda_distill_fwdbwd device status: {_native.status_string(code)}")


class FusedDistillFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, student_hidden, teacher_hidden, weight, teacher_weight, labels, teacher_logits, spec: FusedSpec):
        pr = prepare_call(student_hidden, teacher_hidden, weight, teacher_weight, labels, teacher_logits, spec)
        launch_prepared(pr, spec, keep_alive=ctx)
        out, status = pr.out, pr.status
        g_hs, g_ht, g_w, g_wt, h_t = pr.g_hs, pr.g_ht, pr.g_w, pr.g_wt, pr.h_t

        loss = out[_native.OUT_LOSS].clone()
        ce_s = out[_native.OUT_STUDENT_CE].clone()
        ce_t = out[_native.OUT_TEACHER_CE].clone()
        kl = out[_native.OUT_KL].clone()
        mean_scale = out[_native.OUT_MEAN_SCALE].clone()

        ctx.save_for_backward(g_hs, g_ht, g_w, g_wt, mean_scale, status)
        ctx.shapes = (student_hidden.shape[1], h_t)
        ctx.dtypes = (
            student_hidden.dtype,
            teacher_hidden.dtype if teacher_hidden is not None else None,
            weight.dtype,
            teacher_weight.dtype if teacher_weight is not None else None,
        )
        ctx.mark_non_differentiable(ce_s, ce_t, kl)
        return loss, ce_s, ce_t, kl

    @staticmethod
    @once_differentiable
    def backward(ctx, grad_output, _g1=None, _g2=None, _g3=None):
        g_hs, g_ht, g_w, g_wt, _mean_scale, _status = ctx.saved_tensors
        if grad_output is None:
            return (None,) * 7
        h, h_t = ctx.shapes
        dt_hs, dt_ht, dt_w, dt_wt = ctx.dtypes
        r = rescale_saved_grads(ctx, [(g_hs, h, dt_hs), (g_ht, h_t, dt_ht), (g_w, h, dt_w), (g_wt, h_t, dt_wt)],
                                grad_output)
        return (r[0], r[1], r[2], r[3], None, None, None)


def fused_distillation(
    student_hidden,
    teacher_hidden,
    weight,
    teacher_weight,
    labels,
    teacher_logits,
    spec: FusedSpec,
):
    if torch.compiler.is_compiling():
        # inside torch.compile the call is the traceable custom op (fake implementation + autograd formula)
        from ._op import compiled_fused_distillation

        return compiled_fused_distillation(student_hidden, teacher_hidden, weight, teacher_weight, labels,
                                           teacher_logits, spec)
    return FusedDistillFunction.apply(student_hidden, teacher_hidden, weight, teacher_weight, labels, teacher_logits, spec)
