"""Multi-GPU forms of the distillation loss (one process per GPU, ``torch.distributed`` over NCCL).

The reference has no distributed code; both forms here are additions that keep the single-GPU
semantics of ``distillation_loss`` (same losses, same gradients as one process holding every row and
the whole lm_head).

* Token sharding (:func:`token_parallel_distillation_loss`): every rank holds its own rows and a full
  lm_head replica. The fused kernel runs on the local rows with sum reduction; the loss sums and the
  non-ignored label count are all-reduced (a few bytes) so the returned loss and every gradient use the
  GLOBAL mean. The lm_head gradient of each rank is its local contribution: sum it over ranks (DDP does,
  or :func:`allreduce_weight_grad`).

* Vocab sharding (:func:`vocab_parallel_distillation_loss`): every rank holds all rows and a slice of
  the lm_head rows (vocab ids ``vocab_offset .. vocab_offset + V_local``). Each rank computes the softmax
  statistics of its slice; the per-row records (16 floats per row) are all-gathered and LSE-merged, so
  every rank sees the global log-sum-exps (for JSD the two per-row partial sums are all-reduced as
  well). Each rank then writes its dlogits, its complete lm_head-slice gradient (no communication) and
  a partial hidden-state gradient that is all-reduced.
"""
from __future__ import annotations

import torch
import torch.distributed as dist
from torch.autograd.function import once_differentiable

from . import _native
from ._fused import FusedSpec, prepare_call, rescale_saved_grads
from .api import (
    DistillationLossOutput,
    PrecomputedTeacher,
    SeparateTeacher,
    TiedTeacher,
    _resolve_teacher_ce_weight,
    _teacher_mode_and_tensors,
    distillation_loss,
)
from .ops._common import check_divergence


# ---------------------------------------------------------------------------------- token sharding
def token_parallel_distillation_loss(student_hidden, weight, labels, teacher, *, group=None, reduction="mean",
                                     _local_loss=None, **kwargs) -> DistillationLossOutput:
    """``distillation_loss`` over the rows of all ranks in ``group``; this rank passes its own rows.

    Returns the global loss and components (identical on every rank). Gradients w.r.t. this rank's
    hidden states are final; the lm_head gradient is this rank's share of the global gradient.
    ``_local_loss`` replaces the per-rank loss call (tests inject a CPU formula).
    """
    if reduction not in ("mean", "sum"):
        raise ValueError(f"reduction must be 'mean' or 'sum', got {reduction!r}")
    local = _local_loss or distillation_loss
    out = local(student_hidden, weight, labels, teacher, reduction="sum", **kwargs)
    ignore_index = kwargs.get("ignore_index", -100)
    count = (labels != ignore_index).sum().to(torch.float32)
    stats = torch.stack([out.loss.detach().float(), out.student_ce.float(), out.teacher_ce.float(),
                         out.kl.float(), count.to(out.loss.device)])
    dist.all_reduce(stats, group=group)
    inv = 1.0 / torch.clamp(stats[4], min=1.0) if reduction == "mean" else torch.ones((), device=stats.device)
    # global loss: this rank's sum carries the gradient, the other ranks' sums are constants
    loss = out.loss * inv + (stats[0] - out.loss.detach()) * inv
    return DistillationLossOutput(loss, stats[1] * inv, stats[2] * inv, stats[3] * inv)


class PeerGradientExchange:
    """Sums the lm_head gradient of token-sharded data parallelism over the ranks through peer memory
    (NVLink), instead of an NCCL all-reduce of the whole [V, H] gradient.

    Rank r owns lm_head rows ``[r * slab, (r + 1) * slab)``. Two buffers per rank are mapped into every
    peer's address space (CUDA IPC through ``orda_ipc_export`` / ``orda_ipc_import``): ``slots`` ([world * slab, H]; slot k receives rank k's
    partial gradient of this rank's rows) and ``grad`` ([V, H], the summed gradient). Per step:

    1. the fused call's dW GEMM stores each row of this rank's partial gradient into its owner's slot
       from the GEMM epilogue (``orda_distill_fwdbwd_peer``), overlapped with the GEMM's other tiles;
       the dHidden GEMM follows on the same stream;
    2. on a side stream, after that GEMM: a one-element NCCL all-reduce (every rank's routed stores
       are done), ``orda_peer_reduce_broadcast`` (this rank sums its slots and writes the sum into every
       rank's ``grad``, beside the dHidden GEMM), and a second one-element all-reduce (every owner has
       written this rank's ``grad``); the current stream then waits for the side stream.

    No kernel waits on another GPU; the two tiny collectives order the phases. The returned lm_head
    gradient is ``grad`` itself, reused by the next step (consume it, e.g. with the optimizer step,
    before the next forward, as with DDP's gradient buckets).
    """

    def __init__(self, weight: torch.Tensor, group=None, reduce_ctas: int = 64):
        import ctypes

        lib = _native.load()
        self.group = group or dist.group.WORLD
        self.world = dist.get_world_size(self.group)
        self.rank = dist.get_rank(self.group)
        if self.world > _native.MAX_PEERS:
            raise ValueError(f"peer gradient exchange supports at most {_native.MAX_PEERS} ranks")
        if weight.dtype not in (torch.bfloat16, torch.float16):
            raise ValueError("peer gradient exchange needs a 16-bit lm_head")
        vocab, hidden = weight.shape
        if hidden % 8:
            raise ValueError("peer gradient exchange needs hidden % 8 == 0")
        dev = weight.device
        self.vocab, self.hidden, self.dtype = vocab, hidden, weight.dtype
        # whole 512-row dW tiles per owner, so the dW epilogue can store routed rows by TMA
        self.slab = -(-(-(-vocab // self.world)) // 512) * 512
        self.slots = torch.empty((self.world * self.slab, hidden), dtype=weight.dtype, device=dev)
        self.grad = torch.empty((vocab, hidden), dtype=weight.dtype, device=dev)
        # every rank maps the other ranks' two buffers (CUDA IPC; plain peer mappings over NVLink)
        mine = []
        for t in (self.slots, self.grad):
            h = _native.IpcHandle()
            _native.check(lib.orda_ipc_export(t.data_ptr(), ctypes.byref(h)), "orda_ipc_export")
            mine.append((bytes(h.handle), int(h.offset)))
        everyone = [None] * self.world
        dist.all_gather_object(everyone, mine, group=self.group)
        d = _native.PeerSlots()
        d.world, d.rank, d.slab_rows = self.world, self.rank, self.slab
        self._imported = []
        for k in range(self.world):
            for i, (local, field) in enumerate(((self.slots, d.slot_base), (self.grad, d.grad_base))):
                if k == self.rank:
                    field[k] = local.data_ptr()
                    continue
                h = _native.IpcHandle()
                ctypes.memmove(h.handle, everyone[k][i][0], 64)
                h.offset = everyone[k][i][1]
                ptr = ctypes.c_void_p()
                _native.check(lib.orda_ipc_import(ctypes.byref(h), ctypes.byref(ptr)), "orda_ipc_import")
                self._imported.append((ptr, h))
                field[k] = ptr.value
        self.desc = d
        self.reduce_ctas = int(reduce_ctas)
        self.comm = torch.cuda.Stream(device=dev)
        self.dweight_done = torch.cuda.Event()
        self.dweight_done.record()  # torch creates the CUDA event on first record; the library records it
        self.finished = torch.cuda.Event()
        self._flag = torch.zeros(1, dtype=torch.float32, device=dev)

    def close(self) -> None:
        """Unmap the peers' buffers after the last step that used them has finished. Every rank
        calls this, then a barrier, before any rank frees its own buffers or exits: an exporter that
        goes away while a peer still maps its memory can stall the teardown."""
        import ctypes

        if not getattr(self, "_imported", None):
            return
        torch.cuda.synchronize(self.grad.device)
        lib = _native.load()
        for ptr, h in self._imported:
            lib.orda_ipc_close(ptr, ctypes.byref(h))
        self._imported = []

    def prepare(self, pr) -> None:
        """Point the fused call at this exchange: its lm_head gradient is ``grad``, the dW GEMM runs
        before the dHidden GEMM and marks its end with ``dweight_done``."""
        if pr.g_w.shape != self.grad.shape or pr.g_w.dtype != self.grad.dtype:
            raise ValueError("peer gradient exchange: lm_head gradient shape/dtype differs from the exchange's")
        pr.g_w = self.grad
        a = pr.args
        a.grad_weight = self.grad.data_ptr()
        a.dweight_first = 1
        a.overlap_reserve_sms = 0
        a.dweight_done_event = self.dweight_done.cuda_event

    def complete(self) -> None:
        """Enqueue phase 2 on the side stream after the routed dW GEMM; the current stream waits for it."""
        lib = _native.load()
        self.comm.wait_event(self.dweight_done)
        with torch.cuda.stream(self.comm):
            dist.all_reduce(self._flag, group=self.group)
            _native.check(lib.orda_peer_reduce_broadcast(self.desc, self.vocab, self.hidden,
                                                         _native.BF16 if self.dtype == torch.bfloat16 else _native.F16,
                                                         self.reduce_ctas, self.comm.cuda_stream),
                          "orda_peer_reduce_broadcast")
            dist.all_reduce(self._flag, group=self.group)
            self.finished.record()
        torch.cuda.current_stream().wait_event(self.finished)


def allreduce_weight_grad(weight: torch.Tensor, group=None, async_op: bool = False):
    """Sum ``weight.grad`` over the ranks of ``group`` (token-sharded data parallelism)."""
    if weight.grad is None:
        return None
    return dist.all_reduce(weight.grad, group=group, async_op=async_op)


# ---------------------------------------------------------------------------------- vocab sharding
class _NativeShardOps:
    """The C-ABI phases of one vocab shard (include/orda_b200.h, orda_shard_*). The sharded Function
    only talks to this interface (prepare / forward / merge / jsd_partials / backward / rescale), so the
    CPU tests can run its collective choreography on gloo ranks with a torch restatement."""

    def __init__(self):
        self.lib = _native.load()

    @staticmethod
    def prepare(*args, **kwargs):
        return prepare_call(*args, **kwargs)

    @staticmethod
    def rescale(ctx, grads, grad_output):
        return rescale_saved_grads(ctx, grads, grad_output)

    def forward(self, pr):
        lib = self.lib
        n = pr.args.n_rows
        ws_bytes = int(lib.orda_shard_workspace_bytes(pr.args))
        self.ws = torch.empty(max(ws_bytes, 256), dtype=torch.uint8, device=pr.dev)
        self.ws_bytes = ws_bytes
        self.stream = torch.cuda.current_stream(pr.dev).cuda_stream
        rs = torch.empty((n, _native.ROW_STATS), dtype=torch.float32, device=pr.dev)
        _native.check(lib.orda_shard_forward(pr.args, self.ws.data_ptr(), ws_bytes, rs.data_ptr(), self.stream),
                      "orda_shard_forward")
        return rs

    def merge(self, gathered, world, n):
        rs = torch.empty((n, _native.ROW_STATS), dtype=torch.float32, device=gathered.device)
        _native.check(self.lib.orda_merge_row_stats(gathered.data_ptr(), world, n, rs.data_ptr(), self.stream),
                      "orda_merge_row_stats")
        return rs

    def jsd_partials(self, pr, row_stats):
        sums = torch.empty((pr.args.n_rows, 2), dtype=torch.float32, device=pr.dev)
        _native.check(self.lib.orda_shard_jsd_partials(pr.args, self.ws.data_ptr(), self.ws_bytes, row_stats.data_ptr(),
                                                        sums.data_ptr(), self.stream), "orda_shard_jsd_partials")
        return sums

    def backward(self, pr, row_stats, row_sums):
        _native.check(self.lib.orda_shard_backward(pr.args, self.ws.data_ptr(), self.ws_bytes, row_stats.data_ptr(),
                                                   None if row_sums is None else row_sums.data_ptr(), self.stream),
                      "orda_shard_backward")

    def release(self):
        self.ws = None


def _check_shard_status(pr, group) -> None:
    """Raise on every rank if any rank's kernels reported a device error (a bounded pipeline wait
    that timed out, or an out-of-range label under validation). The status words are combined with
    a MAX all-reduce first, so no rank returns garbage gradients or is left waiting in a later
    collective while another rank raises."""
    status = getattr(pr, "status", None)
    if status is None:
        return
    word = status.reshape(1).to(torch.int32).clone()
    dist.all_reduce(word, op=dist.ReduceOp.MAX, group=group)
    code = int(word.item())
    if code != _native.OK:
        raise RuntimeError(f"vocab-sharded distillation: device status on some rank: {_native.status_string(code)}")


def _all_gather_records(local: torch.Tensor, world: int, group) -> torch.Tensor:
    """[world, n, ROW_STATS] gather of every rank's row records (one collective on NCCL; the list form
    on backends without the single-tensor gather)."""
    if dist.get_backend(group) == "nccl":
        gathered = torch.empty((world, *local.shape), dtype=local.dtype, device=local.device)
        dist.all_gather_into_tensor(gathered, local, group=group)
        return gathered
    parts = [torch.empty_like(local) for _ in range(world)]
    dist.all_gather(parts, local, group=group)
    return torch.stack(parts)


class _VocabShardFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, student_hidden, teacher_hidden, weight, teacher_weight, labels, teacher_logits, spec,
                vocab_offset, vocab_total, group, ops_factory):
        world = dist.get_world_size(group)
        ops = ops_factory()
        pr = ops.prepare(student_hidden, teacher_hidden, weight, teacher_weight, labels, teacher_logits, spec,
                         vocab_offset=vocab_offset, vocab_total=vocab_total)
        n = pr.args.n_rows
        local = ops.forward(pr)
        gathered = _all_gather_records(local, world, group)
        row_stats = ops.merge(gathered, world, n)
        row_sums = None
        jsd = spec.kl_weight != 0.0 and spec.divergence == "jsd" and 0.0 < spec.jsd_beta < 1.0
        if jsd:
            row_sums = ops.jsd_partials(pr, row_stats)
            dist.all_reduce(row_sums, group=group)
        ops.backward(pr, row_stats, row_sums)
        # The workspace holds this shard's n_rows x V_local logits; nothing after the backward phase
        # reads it, so it goes back to the allocator now rather than living as long as the graph.
        release = getattr(ops, "release", None)
        if release is not None:
            release()
        _check_shard_status(pr, group)
        # The hidden-state gradients are sums over the vocab shards. Each rank's partial is in the
        # compute dtype (one rounding per partial, like the single-GPU path's 16-bit output) and the
        # collective sums those partials.
        for g in (pr.g_hs, pr.g_ht):
            if g is not None:
                dist.all_reduce(g, group=group)
        out = pr.out
        loss = out[_native.OUT_LOSS].clone()
        ce_s, ce_t, kl = (out[i].clone() for i in (_native.OUT_STUDENT_CE, _native.OUT_TEACHER_CE, _native.OUT_KL))
        ctx.save_for_backward(pr.g_hs, pr.g_ht, pr.g_w, pr.g_wt, out[_native.OUT_MEAN_SCALE].clone())
        ctx.rescale = ops.rescale  # only the (static) rescale is needed later, not the shard's buffers
        ctx.shapes = (student_hidden.shape[1], pr.h_t)
        ctx.dtypes = (student_hidden.dtype, teacher_hidden.dtype if teacher_hidden is not None else None,
                      weight.dtype, teacher_weight.dtype if teacher_weight is not None else None)
        ctx.mark_non_differentiable(ce_s, ce_t, kl)
        return loss, ce_s, ce_t, kl

    @staticmethod
    @once_differentiable
    def backward(ctx, grad_output, *_):
        g_hs, g_ht, g_w, g_wt, _mean_scale = ctx.saved_tensors
        if grad_output is None:
            return (None,) * 11
        h, h_t = ctx.shapes
        dt_hs, dt_ht, dt_w, dt_wt = ctx.dtypes
        r = ctx.rescale(ctx, [(g_hs, h, dt_hs), (g_ht, h_t, dt_ht), (g_w, h, dt_w), (g_wt, h_t, dt_wt)],
                            grad_output)
        return (r[0], r[1], r[2], r[3], None, None, None, None, None, None, None)


def vocab_parallel_distillation_loss(student_hidden, weight_shard, labels, teacher, *, vocab_offset: int,
                                     vocab_total: int, group=None, student_ce_weight: float = 1.0,
                                     teacher_ce_weight: float | None = None, kl_weight: float = 0.0,
                                     kl_temperature: float = 1.0, ignore_index: int = -100, reduction: str = "mean",
                                     kl_divergence: str = "forward", jsd_beta: float = 0.5,
                                     fp32_grad_weight_accumulation: bool = False,
                                     _shard_ops=None) -> DistillationLossOutput:
    """``distillation_loss`` with the lm_head split by vocabulary rows across the ranks of ``group``.

    ``weight_shard`` holds vocab ids ``[vocab_offset, vocab_offset + weight_shard.shape[0])`` of a
    ``vocab_total``-row lm_head; a ``SeparateTeacher`` carries the same slice of the teacher lm_head and a
    ``PrecomputedTeacher(logits=...)`` the same columns of the teacher logits. Every rank passes all rows
    and the same labels (global vocab ids). Returns the global loss (identical on every rank); the
    gradient of ``weight_shard`` is the complete gradient of that slice. ``_shard_ops`` replaces the
    per-shard library phases (tests run the collectives on CPU ranks with a torch restatement).
    """
    if reduction not in ("mean", "sum"):
        raise ValueError(f"reduction must be 'mean' or 'sum', got {reduction!r}")
    if kl_temperature <= 0.0:
        raise ValueError(f"kl_temperature must be > 0.0, got {kl_temperature}")
    check_divergence(kl_divergence, jsd_beta)
    mode, th, tw, tl = _teacher_mode_and_tensors(teacher)
    tce = _resolve_teacher_ce_weight(mode, teacher_ce_weight)
    if mode == "precomputed":
        if tce != 0.0:
            raise ValueError("PrecomputedTeacher requires teacher_ce_weight=0.0")
        mode = "precomputed_logits" if tl is not None else "precomputed_hidden"
    if not (0 <= vocab_offset and vocab_offset + weight_shard.shape[0] <= vocab_total):
        raise ValueError("weight_shard must lie inside [0, vocab_total)")
    spec = FusedSpec(mode=mode, student_ce_weight=float(student_ce_weight), teacher_ce_weight=float(tce),
                     kl_weight=float(kl_weight), kl_temperature=float(kl_temperature), ignore_index=int(ignore_index),
                     reduction=reduction, divergence=kl_divergence, jsd_beta=float(jsd_beta),
                     fp32_grad_weight=bool(fp32_grad_weight_accumulation))
    if isinstance(teacher, (TiedTeacher, SeparateTeacher, PrecomputedTeacher)) is False:
        raise TypeError("teacher must be TiedTeacher, SeparateTeacher, or PrecomputedTeacher")
    out = _VocabShardFunction.apply(student_hidden, th, weight_shard, tw, labels, tl, spec, int(vocab_offset),
                                    int(vocab_total), group, _shard_ops or _NativeShardOps)
    return DistillationLossOutput(*out)
