"""The op surface of the reference extension module ``mask_loss``.

Same op names, positional argument order, meaning and return values as the
``PYBIND11_MODULE`` in src/bindings.cpp:157-169 of AndyBarcia/mask_loss, so
``sys.modules["mask_loss"] = mask_loss_b200.ops`` makes the reference's own
``functions/`` wrappers run on this implementation.  Argument checks raise
``RuntimeError`` with the reference's TORCH_CHECK messages.

Every op runs on ``torch.cuda.current_stream()`` through the C ABI of
``libmask_loss_b200.so``; there is no CPU path.  Nothing here synchronises the
device: the assignment solver's failure flag is checked without blocking (the
next op call, or :func:`check_status`, raises if an earlier solve failed), and
``MASK_LOSS_B200_SYNC_CHECK=1`` makes every call check it synchronously.
"""
from __future__ import annotations

import ctypes
import os
from typing import List, Optional

import torch

from . import _lib

_SYNC = os.environ.get("MASK_LOSS_B200_SYNC_CHECK", "0") == "1"
_pending: list = []  # (event, pinned int32 flag, message) of earlier device checks


def _lib_handle():
    return _lib.load()


def _ptr(t: Optional[torch.Tensor]):
    # a plain int (or None for NULL): ctypes converts it for the c_void_p
    # arguments the bindings declare
    return t.data_ptr() if t is not None else None


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def _stream_handle(device) -> int:
    if _raw_stream is not None:
        return _raw_stream(device.index if device.index is not None else torch.cuda.current_device())
    return torch.cuda.current_stream(device).cuda_stream


def _stream(device) -> int:
    return _stream_handle(device)


def _check_input(t: torch.Tensor, name: str) -> None:
    if not t.is_cuda:
        raise RuntimeError(f"{name} must be a CUDA tensor")
    if not t.is_contiguous():
        raise RuntimeError(f"{name} must be contiguous")


def _check_dtype(t: torch.Tensor, dtype, name: str) -> None:
    if t.dtype != dtype:
        raise RuntimeError(f"{name} must be {str(dtype).replace('torch.', '')}")


def check_status(block: bool = False) -> None:
    """Raise if an earlier on-device assignment solve reported failure."""
    if torch.cuda.is_available() and torch.cuda.is_current_stream_capturing():
        return  # no event queries inside stream capture
    for st in list(_sticky.values()):
        st.check(block)
    if block and torch.cuda.is_available() and _lib.loaded():
        # the cost-only ops' word (they have no per-call status argument)
        v = ctypes.c_int32(0)
        _lib.check(_lib.load().ml_cost_status(ctypes.byref(v)))
        if v.value:
            raise RuntimeError(_status_message(v.value))
    keep = []
    err = None
    for ev, host, msg in _pending:
        if block:
            ev.synchronize()
        if ev.query():
            v = int(host.item())
            if v != 0 and err is None:
                err = RuntimeError(msg(v) if callable(msg) else msg)
            _pinned.append(host)
        else:
            keep.append((ev, host, msg))
    _pending[:] = keep
    if err is not None:
        raise err


_captured: list = []  # (device int32 flag, message) recorded during stream capture
_pinned = []  # pool of 1-element pinned int32 buffers, reused once their event completed


def _pinned_slot() -> torch.Tensor:
    if _pinned:
        return _pinned.pop()
    return torch.empty(1, dtype=torch.int32, pin_memory=True)


def _defer(flag_i32: torch.Tensor, message: str) -> None:
    if torch.cuda.is_current_stream_capturing():
        # inside CUDA-graph capture: the flag stays on the device; the graph's
        # owner (graphs.MatchingLossStep) checks it after replays
        _captured.append((flag_i32, message))
        return
    if len(_pending) > 64:
        check_status()
    host = _pinned_slot()
    host.copy_(flag_i32, non_blocking=True)
    ev = torch.cuda.Event()
    ev.record(torch.cuda.current_stream(flag_i32.device))
    _pending.append((ev, host, message))
    if _SYNC:
        check_status(block=True)


def defer_check(flag: torch.Tensor, message: str) -> None:
    """Raise ``message`` from a later op call (or check_status) if the device
    boolean ``flag`` is true -- argument checks without a host sync."""
    _defer(flag.reshape(1).to(torch.int32), message)


def _status_message(v: int) -> str:
    if v & 4:
        return "cls_targets must not contain the void class index"
    if v & 2:
        return "mask_loss_b200: a device wait timed out (cost kernel pipeline)"
    return "Hungarian: no augmenting path found; check costs/inf_thresh."


def _track_status(status: torch.Tensor) -> None:
    _defer(status, _status_message)


# ---------------------------------------------------------------------------
# Per-stream state of the two hot ops (outside CUDA-graph capture): a sticky
# device status word that the kernels OR their error bits into, read back
# every _STATUS_EVERY calls (and by check_status); and the scratch workspace,
# reused by every call on the same stream (stream order keeps calls apart).
# ---------------------------------------------------------------------------
_STATUS_EVERY = 8


class _StickyStatus:
    def __init__(self, device):
        self.dev = torch.zeros(1, dtype=torch.int32, device=device)
        self.host = torch.zeros(1, dtype=torch.int32, pin_memory=True)
        self.ev = torch.cuda.Event()
        self.stream = torch.cuda.current_stream(device)
        self.inflight = False
        self.calls = 0

    def after_call(self):
        self.calls += 1
        if self.inflight and self.ev.query():
            self._consume()
        if not self.inflight and (_SYNC or self.calls % _STATUS_EVERY == 0):
            self._issue()
        if _SYNC:
            self.check(block=True)

    def _issue(self):
        self.host.copy_(self.dev, non_blocking=True)
        self.ev.record(self.stream)
        self.inflight = True

    def _consume(self):
        self.inflight = False
        v = int(self.host[0])
        if v != 0:
            with torch.cuda.stream(self.stream):
                self.dev.zero_()
            self.host.zero_()
            raise RuntimeError(_status_message(v))

    def check(self, block: bool):
        if block and not self.inflight:
            self._issue()
        if self.inflight:
            if block:
                self.ev.synchronize()
            if self.ev.query():
                self._consume()


_sticky: dict = {}
_ws_cache: dict = {}
_fwd_plans: dict = {}  # argument key -> (ml_dims, ml_params, GT_out, workspace bytes)
_bwd_plans: dict = {}


def _stream_key(device):
    return (device.index, _stream_handle(device))


def _sticky_status(device) -> Optional[_StickyStatus]:
    """The stream's sticky status word, or None inside stream capture."""
    if torch.cuda.is_current_stream_capturing():
        return None
    k = _stream_key(device)
    st = _sticky.get(k)
    if st is None:
        st = _sticky[k] = _StickyStatus(device)
    return st


def _cached_workspace(nbytes: int, device, tag: str) -> torch.Tensor:
    """A workspace of at least nbytes reused by every call on this stream;
    a fresh one inside stream capture."""
    if torch.cuda.is_current_stream_capturing():
        return _workspace(nbytes, device)
    k = _stream_key(device) + (tag,)
    ws = _ws_cache.get(k)
    if ws is None or ws.numel() < nbytes:
        ws = _ws_cache[k] = _workspace(nbytes, device)
    return ws


def _params(smooth=1.0, sigmoid_scale=1.0, dice_scale=1.0, cls_scale=1.0, background_index=-1,
            uncertainty_gamma=1.0, uncertainty_gamma_min=0.05, inf_thresh=1e30, num_masks=-1.0,
            force_unmatched_class_to_background=False, force_unmatched_masks_to_empty=False,
            topk_matches=1, strategy_id=0, mask_gamma=0.0, mask_alpha=-1.0, cls_gamma=0.0,
            cls_alpha=-1.0, void_class_index=-1, use_softmax_label_loss=False,
            normalize_uncertainty=True, check_void_targets=False) -> _lib.Params:
    return _lib.Params(float(smooth), float(sigmoid_scale), float(dice_scale), float(cls_scale),
                       int(background_index), float(uncertainty_gamma),
                       float(uncertainty_gamma_min), float(inf_thresh), float(num_masks),
                       int(bool(force_unmatched_class_to_background)),
                       int(bool(force_unmatched_masks_to_empty)), int(topk_matches),
                       int(strategy_id), float(mask_gamma), float(mask_alpha), float(cls_gamma),
                       float(cls_alpha), int(void_class_index), int(bool(use_softmax_label_loss)),
                       int(bool(normalize_uncertainty)), int(bool(check_void_targets)))


def is_dense(mask_targets) -> bool:
    """Dense per-GT masks (B, GT_total, H_t, W_t) uint8/bool instead of a
    (B, H_t, W_t) label map (no reference counterpart; overlap allowed)."""
    return mask_targets.dim() == 4


def _dims(mask_logits, mask_targets, cls_logits, cls_targets) -> _lib.Dims:
    L, B, Q, H, W = mask_logits.shape
    Ht, Wt = mask_targets.shape[-2:]
    return _lib.Dims(L, B, Q, H, W, Ht, Wt, cls_logits.shape[3], cls_targets.shape[1])


# mask-logit element types of the label-map entries (ml_params.logits_dtype)
_LOGIT_DTYPES = {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}


def _with_dtype(p: _lib.Params, mask_logits: torch.Tensor) -> _lib.Params:
    p.logits_dtype = _LOGIT_DTYPES[mask_logits.dtype]
    return p


def _check_quad(mask_logits, mask_targets, cls_logits, cls_targets):
    for t, n in ((mask_logits, "mask_logits"), (mask_targets, "mask_targets"),
                 (cls_logits, "cls_logits"), (cls_targets, "cls_targets")):
        _check_input(t, n)
    if mask_logits.dim() != 5:
        raise RuntimeError("mask_logits must be (L,B,Q,H,W)")
    if mask_targets.dim() not in (3, 4):
        raise RuntimeError("mask_targets must be (B,H_t,W_t) labels or (B,GT,H_t,W_t) masks")
    if cls_logits.dim() != 4:
        raise RuntimeError("cls_logits must be (L,B,Q,C)")
    if cls_targets.dim() != 2:
        raise RuntimeError("cls_targets must be (B,GT)")
    if mask_logits.dtype not in _LOGIT_DTYPES:
        raise RuntimeError("mask_logits must be float32, bfloat16 or float16")
    _check_dtype(cls_logits, torch.float32, "cls_logits")
    if is_dense(mask_targets):
        if mask_targets.dtype not in (torch.uint8, torch.bool):
            raise RuntimeError("dense mask_targets must be uint8 or bool")
        if mask_targets.shape[1] != cls_targets.shape[1]:
            raise RuntimeError("dense mask_targets must have one mask per cls_targets column")
    else:
        _check_dtype(mask_targets, torch.int64, "mask_targets")
    _check_dtype(cls_targets, torch.int64, "cls_targets")
    L, B, Q = mask_logits.shape[:3]
    if mask_targets.shape[0] != B or cls_targets.shape[0] != B:
        raise RuntimeError("batch size mismatch between logits and targets")
    if tuple(cls_logits.shape[:3]) != (L, B, Q):
        raise RuntimeError("cls_logits must match mask logits dimensions")


def _workspace(nbytes: int, device) -> torch.Tensor:
    return torch.empty(max(int(nbytes), 1), dtype=torch.uint8, device=device)


# ---------------------------------------------------------------------------
# pairwise_mask_loss_forward (src/bindings.cpp:64-82)
# ---------------------------------------------------------------------------
def pairwise_mask_loss_forward(mask_logits, mask_targets, cls_logits, cls_targets, smooth,
                               sigmoid_scale=1.0, dice_scale=1.0, cls_scale=1.0,
                               background_index=-1, uncertainty_gamma=1.0,
                               uncertainty_gamma_min=0.05, mask_gamma=0.0, mask_alpha=-1.0,
                               cls_gamma=0.0, cls_alpha=-1.0, use_softmax_label_loss=False,
                               normalize_uncertainty=True) -> torch.Tensor:
    """(3,L,B,Q,GT_out) sigmoid-CE, dice and label costs; (L,B,Q,0) when no
    column is left (src/cuda/pw_mask.cu:396-398)."""
    _check_quad(mask_logits, mask_targets, cls_logits, cls_targets)
    lib = _lib_handle()
    d = _dims(mask_logits, mask_targets, cls_logits, cls_targets)
    p = _params(smooth, sigmoid_scale, dice_scale, cls_scale, background_index, uncertainty_gamma,
                uncertainty_gamma_min, mask_gamma=mask_gamma, mask_alpha=mask_alpha,
                cls_gamma=cls_gamma, cls_alpha=cls_alpha,
                use_softmax_label_loss=use_softmax_label_loss,
                normalize_uncertainty=normalize_uncertainty)
    _with_dtype(p, mask_logits)
    L, B, Q = mask_logits.shape[:3]
    G = lib.ml_gt_out(d.GT_total, p.background_index)
    if G == 0:
        return torch.zeros((L, B, Q, 0), dtype=torch.float32, device=mask_logits.device)
    out = torch.empty((3, L, B, Q, G), dtype=torch.float32, device=mask_logits.device)
    dense = is_dense(mask_targets)
    size_fn = lib.ml_dense_workspace_size if dense else lib.ml_mask_matching_workspace_size
    nbytes = size_fn(ctypes.byref(d), ctypes.byref(p))
    if nbytes == 0:
        raise RuntimeError(lib.ml_last_error().decode() or "invalid shapes")
    ws = _workspace(nbytes, mask_logits.device)
    fn = lib.ml_pairwise_mask_loss_dense_forward if dense else lib.ml_pairwise_mask_loss_forward
    _lib.check(fn(ctypes.byref(d), ctypes.byref(p), _ptr(mask_logits), _ptr(mask_targets),
                  _ptr(cls_logits), _ptr(cls_targets), _ptr(out), _ptr(ws), ws.numel(),
                  _stream(mask_logits.device)))
    return out


# ---------------------------------------------------------------------------
# mask_matching (src/bindings.cpp:86-111) and its extended form
# ---------------------------------------------------------------------------
def mask_matching_ex(mask_logits, mask_targets, cls_logits, cls_targets, smooth,
                     sigmoid_scale=1.0, dice_scale=1.0, cls_scale=1.0, background_index=-1,
                     uncertainty_gamma=1.0, uncertainty_gamma_min=0.05, inf_thresh=1e30,
                     num_masks=-1.0, force_unmatched_class_to_background=False,
                     force_unmatched_masks_to_empty=False, topk_matches=1, strategy_id=0,
                     mask_gamma=0.0, mask_alpha=-1.0, cls_gamma=0.0, cls_alpha=-1.0,
                     void_class_index=-1, use_softmax_label_loss=False, normalize_uncertainty=True,
                     *, num_masks_dev: Optional[torch.Tensor] = None, want_saved: bool = False,
                     want_costs: bool = False, check_void_targets: bool = False,
                     loss_wait_event: Optional[torch.cuda.Event] = None,
                     costs_done_event: Optional[torch.cuda.Event] = None,
                     want_workspace: bool = False):
    """``mask_matching`` plus the extras this implementation offers: a device
    ``num_masks_dev`` (fp32 scalar, e.g. after an all-reduce), the per-query
    statistics the backward can reuse (``saved``) and the cost slices.

    ``check_void_targets``: raise (deferred) if cls_targets holds
    void_class_index -- functions/mask/matching.py:180-181, checked on the
    device.  ``loss_wait_event``: the matched-loss kernel (the only reader
    of ``num_masks_dev``) waits for it, so an all-reduce producing that count
    on another stream overlaps the cost and solver kernels.
    ``costs_done_event``: recorded once the costs are final, before the solver
    (work on another stream may wait for it and run beside the solver).

    ``want_workspace``: also return the forward workspace, which
    mask_matching_backward(forward_workspace=) reuses (label-map targets).

    Returns (pred_to_gt, pred_round, layer_means(3,L), saved or None, costs or None)
    [+ workspace]."""
    check_status()
    _check_quad(mask_logits, mask_targets, cls_logits, cls_targets)
    if topk_matches < 0:
        raise RuntimeError("K must be non-negative")
    if not 0 <= strategy_id <= 3:
        raise RuntimeError("Invalid matching strategy id")
    lib = _lib_handle()
    dev = mask_logits.device
    dense = is_dense(mask_targets)
    key = (mask_logits.shape, mask_logits.dtype, mask_targets.shape, cls_logits.shape,
           cls_targets.shape, smooth, sigmoid_scale, dice_scale, cls_scale, background_index,
           uncertainty_gamma, uncertainty_gamma_min, inf_thresh, num_masks,
           force_unmatched_class_to_background, force_unmatched_masks_to_empty, topk_matches,
           strategy_id, mask_gamma, mask_alpha, cls_gamma, cls_alpha, void_class_index,
           use_softmax_label_loss, normalize_uncertainty, check_void_targets)
    plan = _fwd_plans.get(key)
    if plan is None:
        d = _dims(mask_logits, mask_targets, cls_logits, cls_targets)
        p = _params(smooth, sigmoid_scale, dice_scale, cls_scale, background_index,
                    uncertainty_gamma, uncertainty_gamma_min, inf_thresh, num_masks,
                    force_unmatched_class_to_background, force_unmatched_masks_to_empty,
                    topk_matches, strategy_id, mask_gamma, mask_alpha, cls_gamma, cls_alpha,
                    void_class_index, use_softmax_label_loss, normalize_uncertainty,
                    check_void_targets)
        _with_dtype(p, mask_logits)
        size_fn = lib.ml_dense_workspace_size if dense else lib.ml_mask_matching_workspace_size
        nb = size_fn(ctypes.byref(d), ctypes.byref(p))
        if nb == 0:
            raise RuntimeError(lib.ml_last_error().decode() or "invalid shapes")
        plan = (d, p, lib.ml_gt_out(d.GT_total, p.background_index), nb)
        if len(_fwd_plans) > 256:
            _fwd_plans.clear()
        _fwd_plans[key] = plan
    d, p, G, nbytes = plan
    L, B, Q = mask_logits.shape[:3]
    LBQ = L * B * Q
    idx = torch.empty((2, L, B, Q), dtype=torch.int64, device=dev)
    p2g, prd = idx[0], idx[1]
    fl = torch.empty(3 * L + (4 * LBQ if want_saved else 0), dtype=torch.float32, device=dev)
    means = fl[:3 * L].view(3, L)
    saved = fl[3 * L:].view(L, B, Q, 4) if want_saved else None
    costs = (torch.empty((3, L, B, Q, G), dtype=torch.float32, device=dev)
             if want_costs and G > 0 else None)
    sticky = _sticky_status(dev)
    status = sticky.dev if sticky is not None else torch.zeros(1, dtype=torch.int32, device=dev)
    # the forward workspace is handed out when asked for (its codes feed the
    # backward), otherwise the stream's cached one is used
    ws = _workspace(nbytes, dev) if want_workspace else _cached_workspace(nbytes, dev, "fwd")
    if num_masks_dev is not None:
        _check_input(num_masks_dev, "num_masks_dev")
        _check_dtype(num_masks_dev, torch.float32, "num_masks_dev")
    if dense:
        if loss_wait_event is not None or costs_done_event is not None:
            raise RuntimeError("stream events are not supported with dense mask targets")
        _lib.check(lib.ml_mask_matching_dense(
            ctypes.byref(d), ctypes.byref(p), _ptr(mask_logits), _ptr(mask_targets),
            _ptr(cls_logits), _ptr(cls_targets), _ptr(num_masks_dev), _ptr(p2g), _ptr(prd),
            _ptr(means), _ptr(costs), _ptr(saved), _ptr(status), _ptr(ws), ws.numel(),
            _stream(dev)))
    elif costs_done_event is not None:
        if not costs_done_event.cuda_event:
            raise RuntimeError("costs_done_event has no CUDA event yet: record it once first")
        _lib.check(lib.ml_mask_matching_ex2(
            ctypes.byref(d), ctypes.byref(p), _ptr(mask_logits), _ptr(mask_targets),
            _ptr(cls_logits), _ptr(cls_targets), _ptr(num_masks_dev), _ptr(p2g), _ptr(prd),
            _ptr(means), _ptr(costs), _ptr(saved), _ptr(status), _ptr(ws), ws.numel(),
            _stream(dev), ctypes.c_void_p(loss_wait_event.cuda_event if loss_wait_event else 0),
            ctypes.c_void_p(costs_done_event.cuda_event)))
    elif loss_wait_event is not None:
        _lib.check(lib.ml_mask_matching_ex(
            ctypes.byref(d), ctypes.byref(p), _ptr(mask_logits), _ptr(mask_targets),
            _ptr(cls_logits), _ptr(cls_targets), _ptr(num_masks_dev), _ptr(p2g), _ptr(prd),
            _ptr(means), _ptr(costs), _ptr(saved), _ptr(status), _ptr(ws), ws.numel(),
            _stream(dev), ctypes.c_void_p(loss_wait_event.cuda_event)))
    else:
        _lib.check(lib.ml_mask_matching(
            ctypes.byref(d), ctypes.byref(p), _ptr(mask_logits), _ptr(mask_targets),
            _ptr(cls_logits), _ptr(cls_targets), _ptr(num_masks_dev), _ptr(p2g), _ptr(prd),
            _ptr(means), _ptr(costs), _ptr(saved), _ptr(status), _ptr(ws), ws.numel(),
            _stream(dev)))
    if sticky is not None:
        sticky.after_call()
    else:
        _track_status(status)
    if want_workspace:
        return p2g, prd, means, saved, costs, ws
    return p2g, prd, means, saved, costs


def mask_matching(mask_logits, mask_targets, cls_logits, cls_targets, smooth, sigmoid_scale=1.0,
                  dice_scale=1.0, cls_scale=1.0, background_index=-1, uncertainty_gamma=1.0,
                  uncertainty_gamma_min=0.05, inf_thresh=1e30, num_masks=-1.0,
                  force_unmatched_class_to_background=False, force_unmatched_masks_to_empty=False,
                  topk_matches=1, strategy_id=0, mask_gamma=0.0, mask_alpha=-1.0, cls_gamma=0.0,
                  cls_alpha=-1.0, void_class_index=-1, use_softmax_label_loss=False,
                  normalize_uncertainty=True) -> List[torch.Tensor]:
    """[pred_to_gt, pred_round, layer_mask_mean, layer_dice_mean, layer_cls_mean]
    (src/cpu/matching.cpp:592-752)."""
    p2g, prd, means, _, _ = mask_matching_ex(
        mask_logits, mask_targets, cls_logits, cls_targets, smooth, sigmoid_scale, dice_scale,
        cls_scale, background_index, uncertainty_gamma, uncertainty_gamma_min, inf_thresh,
        num_masks, force_unmatched_class_to_background, force_unmatched_masks_to_empty,
        topk_matches, strategy_id, mask_gamma, mask_alpha, cls_gamma, cls_alpha, void_class_index,
        use_softmax_label_loss, normalize_uncertainty)
    return [p2g, prd, means[0], means[1], means[2]]


# ---------------------------------------------------------------------------
# mask_matching_backward (src/bindings.cpp:113-139)
# ---------------------------------------------------------------------------
def mask_matching_backward(grad_layer_mask_mean, grad_layer_dice_mean, grad_layer_cls_mean,
                           mask_logits, mask_targets, cls_logits, cls_targets, pred_to_gt,
                           smooth, sigmoid_scale, dice_scale, cls_scale, background_index,
                           uncertainty_gamma, uncertainty_gamma_min, num_masks,
                           force_unmatched_class_to_background, force_unmatched_masks_to_empty,
                           mask_gamma, mask_alpha, cls_gamma, cls_alpha, void_class_index,
                           use_softmax_label_loss=False, normalize_uncertainty=True, *,
                           saved: Optional[torch.Tensor] = None,
                           num_masks_dev: Optional[torch.Tensor] = None,
                           forward_workspace: Optional[torch.Tensor] = None,
                           grad_mask_out: Optional[torch.Tensor] = None,
                           grad_rows_prezeroed: bool = False) -> List[torch.Tensor]:
    """[grad_mask_logits, grad_cls_logits] (src/cuda/mask_matching_backward.cu:378-621).

    ``forward_workspace``: the workspace returned by mask_matching_ex(want_workspace=True)
    for the same inputs and arguments; its per-cell label codes are reused.
    ``grad_mask_out``: the buffer to write the mask gradient into (like
    mask_logits); with ``grad_rows_prezeroed`` the caller has filled it with
    zeros and only the rows that carry a gradient are written."""
    check_status()
    for t, n in ((grad_layer_mask_mean, "grad_layer_mask_mean"),
                 (grad_layer_dice_mean, "grad_layer_dice_mean"),
                 (grad_layer_cls_mean, "grad_layer_cls_mean"), (pred_to_gt, "pred_to_gt")):
        _check_input(t, n)
    _check_quad(mask_logits, mask_targets, cls_logits, cls_targets)
    _check_dtype(grad_layer_mask_mean, torch.float32, "grad_layer_mask_mean")
    _check_dtype(grad_layer_dice_mean, torch.float32, "grad_layer_dice_mean")
    _check_dtype(grad_layer_cls_mean, torch.float32, "grad_layer_cls_mean")
    _check_dtype(pred_to_gt, torch.int64, "pred_to_gt")
    lib = _lib_handle()
    dev = mask_logits.device
    key = (mask_logits.shape, mask_logits.dtype, mask_targets.shape, cls_logits.shape,
           cls_targets.shape, smooth, sigmoid_scale, dice_scale, cls_scale, background_index,
           uncertainty_gamma, uncertainty_gamma_min, num_masks,
           force_unmatched_class_to_background, force_unmatched_masks_to_empty, mask_gamma,
           mask_alpha, cls_gamma, cls_alpha, void_class_index, use_softmax_label_loss,
           normalize_uncertainty)
    plan = _bwd_plans.get(key)
    if plan is None:
        d = _dims(mask_logits, mask_targets, cls_logits, cls_targets)
        p = _params(smooth, sigmoid_scale, dice_scale, cls_scale, background_index,
                    uncertainty_gamma, uncertainty_gamma_min, 1e30, num_masks,
                    force_unmatched_class_to_background, force_unmatched_masks_to_empty, 1, 0,
                    mask_gamma, mask_alpha, cls_gamma, cls_alpha, void_class_index,
                    use_softmax_label_loss, normalize_uncertainty)
        _with_dtype(p, mask_logits)
        plan = (d, p, lib.ml_mask_matching_backward_workspace_size(ctypes.byref(d),
                                                                   ctypes.byref(p)))
        if len(_bwd_plans) > 256:
            _bwd_plans.clear()
        _bwd_plans[key] = plan
    d, p, nbytes = plan
    if grad_mask_out is not None:
        _check_input(grad_mask_out, "grad_mask_out")
        if grad_mask_out.shape != mask_logits.shape or grad_mask_out.dtype != mask_logits.dtype:
            raise RuntimeError("grad_mask_out must match mask_logits in shape and dtype")
        gm = grad_mask_out
    else:
        if grad_rows_prezeroed:
            raise RuntimeError("grad_rows_prezeroed needs grad_mask_out")
        gm = torch.empty_like(mask_logits)
    gc = torch.empty_like(cls_logits)
    ws = _cached_workspace(nbytes, dev, "bwd")
    if saved is not None:
        _check_input(saved, "saved")
    if is_dense(mask_targets) and saved is None:
        raise RuntimeError("dense mask targets need the forward's saved statistics (saved=)")
    args = (ctypes.byref(d), ctypes.byref(p), _ptr(grad_layer_mask_mean),
            _ptr(grad_layer_dice_mean), _ptr(grad_layer_cls_mean), _ptr(mask_logits),
            _ptr(mask_targets), _ptr(cls_logits), _ptr(cls_targets), _ptr(pred_to_gt),
            _ptr(saved), _ptr(num_masks_dev), _ptr(gm), _ptr(gc), _ptr(ws), ws.numel(),
            _stream(dev))
    if is_dense(mask_targets):
        if grad_rows_prezeroed:
            raise RuntimeError("grad_rows_prezeroed is not supported with dense mask targets")
        _lib.check(lib.ml_mask_matching_dense_backward(*args))
    elif grad_rows_prezeroed:
        if forward_workspace is not None:
            _check_input(forward_workspace, "forward_workspace")
        _lib.check(lib.ml_mask_matching_backward_ex2(*args, _ptr(forward_workspace), 1))
    elif forward_workspace is not None:
        _check_input(forward_workspace, "forward_workspace")
        _lib.check(lib.ml_mask_matching_backward_ex(*args, _ptr(forward_workspace)))
    else:
        _lib.check(lib.ml_mask_matching_backward(*args))
    return [gm, gc]


# ---------------------------------------------------------------------------
# Standalone pairwise ops (src/bindings.cpp:22-31, 51-62, 141-155)
# ---------------------------------------------------------------------------
def _pairwise_mask_only(logits, targets, background_index, which, smooth=1.0, scale=1.0, gamma=0.0,
                        alpha=-1.0, ug=1.0, ugmin=0.05, normalize=True, num_gts=None):
    _check_input(logits, "logits")
    _check_input(targets, "targets")
    if logits.dim() != 5:
        raise RuntimeError("logits must be (L,B,C,H,W)")
    # GT_total = targets.max() + 1 (src/cuda/pw_sigmoid_ce.cu:221-224): the output's
    # width, so a host read as in the reference, unless the caller passes it
    if num_gts is not None:
        gt_total = int(num_gts)
    else:
        gt_total = int(targets.max().item()) + 1 if targets.numel() else 0
    L, B, Q = logits.shape[:3]
    dev = logits.device
    cls_logits = torch.zeros((L, B, Q, 1), dtype=torch.float32, device=dev)
    cls_targets = torch.full((B, max(gt_total, 0)), -1, dtype=torch.int64, device=dev)
    out = pairwise_mask_loss_forward(logits, targets, cls_logits, cls_targets, smooth, scale, scale,
                                     1.0, background_index, ug, ugmin, gamma, alpha, 0.0, -1.0,
                                     False, normalize)
    if out.dim() == 4:
        return out
    return out[which].contiguous()


def forward_pw_sigmoid_ce_loss(logits, targets, background_index=-1, scale=1.0, gamma=0.0,
                               alpha=-1.0, uncertainty_gamma=1.0, uncertainty_gamma_min=0.05,
                               normalize_uncertainty=True, *, num_gts=None):
    """(L,B,C,GT_out) pairwise sigmoid-CE (src/cuda/pw_sigmoid_ce.cu:199-316).

    num_gts (keyword, not in the reference): GT_total = targets.max() + 1 when
    the caller knows it; the op then makes no host read of the targets."""
    return _pairwise_mask_only(logits, targets, background_index, 0, 1.0, scale, gamma, alpha,
                               uncertainty_gamma, uncertainty_gamma_min, normalize_uncertainty,
                               num_gts)


def forward_pw_dice_loss(logits, targets, smooth, background_index=-1, scale=1.0,
                         uncertainty_gamma=1.0, uncertainty_gamma_min=0.05, *, num_gts=None):
    """(L,B,C,GT_out) pairwise dice (src/cuda/pw_dice_loss.cu:111-220); num_gts as
    in forward_pw_sigmoid_ce_loss."""
    return _pairwise_mask_only(logits, targets, background_index, 1, smooth, scale, 0.0, -1.0,
                               uncertainty_gamma, uncertainty_gamma_min, True, num_gts)


def _label_cost(logits, targets, background_index, scale, gamma, alpha, softmax, name):
    _check_input(logits, "logits")
    _check_input(targets, "targets")
    if logits.dim() != 4:
        raise RuntimeError(f"{name}: logits must be (L,B,Q,C)")
    if targets.dim() != 2:
        raise RuntimeError(f"{name}: targets must be (B,GT)")
    L, B, Q, C = logits.shape
    if targets.shape[0] != B:
        raise RuntimeError(f"{name}: batch size mismatch between logits and targets")
    lib = _lib_handle()
    G = lib.ml_gt_out(targets.shape[1], int(background_index))
    if G == 0:
        return torch.zeros((L, B, Q, 0), dtype=torch.float32, device=logits.device)
    z = logits.contiguous().float()
    out = torch.empty((L, B, Q, G), dtype=torch.float32, device=logits.device)
    _lib.check(lib.ml_pairwise_label_loss_forward(
        L, B, Q, C, targets.shape[1], int(background_index), float(scale), float(gamma),
        float(alpha), int(softmax), _ptr(z), _ptr(targets.contiguous()), _ptr(out),
        _stream(logits.device)))
    return out


def forward_pw_sigmoid_label_loss(logits, targets, background_index=-1, scale=1.0, gamma=0.0,
                                  alpha=-1.0):
    """(L,B,Q,GT_out) pairwise sigmoid label cost (src/cuda/pw_sigmoid_label_loss.cu:108-187)."""
    return _label_cost(logits, targets, background_index, scale, gamma, alpha, False,
                       "pairwise_sigmoid_label_loss_forward")


def forward_pw_softmax_label_loss(logits, targets, background_index=-1, scale=1.0):
    """(L,B,Q,GT_out) pairwise softmax label cost (src/cuda/pw_softmax_label_loss.cu:105-174)."""
    return _label_cost(logits, targets, background_index, scale, 0.0, -1.0, True,
                       "pairwise_softmax_label_loss_forward")


def _sem_shape(logits, targets):
    _check_input(logits, "logits")
    _check_input(targets, "targets")
    _check_dtype(logits, torch.float32, "logits")
    _check_dtype(targets, torch.int64, "targets")
    if logits.dim() != 5 or targets.dim() != 3:
        raise RuntimeError("logits must be (L,B,C,H,W) and targets (B,H_t,W_t)")
    if logits.device != targets.device:
        raise RuntimeError("logits and targets must be on the same device")
    L, B, C, H, W = logits.shape
    if targets.shape[0] != B:
        raise RuntimeError("Batch size mismatch between logits and targets")
    return (L, B, C, H, W, targets.shape[1], targets.shape[2])


def forward_sigmoid_ce_loss(logits, targets, num_masks, scale=1.0, gamma=0.0, alpha=-1.0):
    """(L,) per-layer (focal) sigmoid BCE, src/cuda/sigmoid_ce.cu:207-267."""
    shp = _sem_shape(logits, targets)
    lib = _lib_handle()
    out = torch.zeros(shp[0], dtype=torch.float32, device=logits.device)
    nbytes = lib.ml_semantic_workspace_size(*shp, 0)
    if nbytes == 0:
        raise RuntimeError(lib.ml_last_error().decode() or "invalid shapes")
    ws = _workspace(nbytes, logits.device)
    _lib.check(lib.ml_sigmoid_ce_forward(*shp, _ptr(logits), _ptr(targets), float(num_masks),
                                         float(scale), float(gamma), float(alpha), _ptr(out),
                                         _ptr(ws), ws.numel(), _stream(logits.device)))
    return out


def backward_sigmoid_ce_loss(grad_out, logits, targets, num_masks, scale=1.0, gamma=0.0,
                             alpha=-1.0):
    """dL/dlogits of forward_sigmoid_ce_loss, src/cuda/sigmoid_ce.cu:269-332."""
    shp = _sem_shape(logits, targets)
    go = grad_out.contiguous().float()
    _check_input(go, "grad_out")
    grad = torch.empty_like(logits)
    _lib.check(_lib_handle().ml_sigmoid_ce_backward(
        *shp, _ptr(go), _ptr(logits), _ptr(targets), float(num_masks), float(scale), float(gamma),
        float(alpha), _ptr(grad), _stream(logits.device)))
    return grad


def forward_dice_loss(logits, targets, smooth, num_masks, scale=1.0):
    """[loss (L,), int_sum, p_sum, t_sum (L,B,C)], src/cuda/dice_loss.cu:159-223."""
    shp = _sem_shape(logits, targets)
    L, B, C = shp[:3]
    lib = _lib_handle()
    dev = logits.device
    out = torch.zeros(L, dtype=torch.float32, device=dev)
    I = torch.zeros((L, B, C), dtype=torch.float32, device=dev)
    P = torch.zeros((L, B, C), dtype=torch.float32, device=dev)
    T = torch.zeros((L, B, C), dtype=torch.float32, device=dev)
    nbytes = lib.ml_semantic_workspace_size(*shp, 1)
    if nbytes == 0:
        raise RuntimeError(lib.ml_last_error().decode() or "invalid shapes")
    ws = _workspace(nbytes, dev)
    _lib.check(lib.ml_dice_forward(*shp, _ptr(logits), _ptr(targets), float(smooth),
                                   float(num_masks), float(scale), _ptr(out), _ptr(I), _ptr(P),
                                   _ptr(T), _ptr(ws), ws.numel(), _stream(dev)))
    return [out, I, P, T]


def backward_dice_loss(grad_out, logits, targets, int_sum, p_sum, t_sum, smooth, num_masks,
                       scale=1.0):
    """dL/dlogits of forward_dice_loss, src/cuda/dice_loss.cu:225-288."""
    shp = _sem_shape(logits, targets)
    go = grad_out.contiguous().float()
    sums = [t.contiguous().float() for t in (int_sum, p_sum, t_sum)]
    for t, n in zip([go] + sums, ("grad_out", "int_sum", "p_sum", "t_sum")):
        _check_input(t, n)
    grad = torch.empty_like(logits)
    _lib.check(_lib_handle().ml_dice_backward(
        *shp, _ptr(go), _ptr(logits), _ptr(targets), _ptr(sums[0]), _ptr(sums[1]), _ptr(sums[2]),
        float(smooth), float(num_masks), float(scale), _ptr(grad), _stream(logits.device)))
    return grad


# ---------------------------------------------------------------------------
# Solver alone (for bit-exact checks on identical fp64 cost matrices)
# ---------------------------------------------------------------------------
def match_costs(costs: torch.Tensor, inf_thresh=1e30, topk=1, strategy_id=0):
    """Assign every slice of a (..., Q, GT_out) fp32 or fp64 cost tensor on
    the GPU.  Returns (pred_to_gt, pred_round) shaped like costs[..., 0]."""
    _check_input(costs, "costs")
    lib = _lib_handle()
    Q, G = costs.shape[-2:]
    N = costs.numel() // max(Q * G, 1) if Q * G else 0
    p2g = torch.empty(costs.shape[:-1], dtype=torch.int64, device=costs.device)
    prd = torch.empty_like(p2g)
    status = torch.zeros(1, dtype=torch.int32, device=costs.device)
    if costs.dtype == torch.float64:
        rc = lib.ml_match_f64(_ptr(costs), N, Q, G, float(inf_thresh), int(topk), int(strategy_id),
                              _ptr(p2g), _ptr(prd), _ptr(status), _stream(costs.device))
    elif costs.dtype == torch.float32:
        rc = lib.ml_match(_ptr(costs), 1, N, Q, G, float(inf_thresh), int(topk), int(strategy_id),
                          _ptr(p2g), _ptr(prd), _ptr(status), None, 0, _stream(costs.device))
    else:
        raise RuntimeError("costs must be float32 or float64")
    _lib.check(rc)
    _track_status(status)
    return p2g, prd


def count_masks(mask_targets, GT_total: int, background_index: int) -> torch.Tensor:
    """Device fp32 scalar: present non-background GT ids summed over the batch."""
    _check_input(mask_targets, "mask_targets")
    lib = _lib_handle()
    B, Ht, Wt = mask_targets.shape
    d = _lib.Dims(1, B, 1, Ht, Wt, Ht, Wt, 1, GT_total)
    p = _params(background_index=background_index)
    out = torch.empty((), dtype=torch.float32, device=mask_targets.device)
    nbytes = lib.ml_mask_matching_workspace_size(ctypes.byref(d), ctypes.byref(p))
    ws = _workspace(nbytes, mask_targets.device)
    _lib.check(lib.ml_count_masks(ctypes.byref(d), ctypes.byref(p), _ptr(mask_targets), _ptr(out),
                                  _ptr(ws), ws.numel(), _stream(mask_targets.device)))
    return out


# ---------------------------------------------------------------------------
# Point-sampled costs and matching (config 3)
# ---------------------------------------------------------------------------
def _dtype_code(t: torch.Tensor) -> int:
    if t.dtype == torch.float32:
        return 0
    if t.dtype == torch.bfloat16:
        return 1
    raise RuntimeError("mask_logits must be float32 or bfloat16")


def _check_sampled(mask_logits, mask_targets, cls_logits, cls_targets, point_coords):
    for t, n in ((mask_logits, "mask_logits"), (mask_targets, "mask_targets"),
                 (cls_logits, "cls_logits"), (cls_targets, "cls_targets"),
                 (point_coords, "point_coords")):
        _check_input(t, n)
    _dtype_code(mask_logits)
    _check_dtype(cls_logits, torch.float32, "cls_logits")
    if is_dense(mask_targets):
        if mask_targets.dtype not in (torch.uint8, torch.bool):
            raise RuntimeError("dense mask_targets must be uint8 or bool")
        if mask_targets.shape[1] != cls_targets.shape[1]:
            raise RuntimeError("dense mask_targets must have one mask per cls_targets column")
    else:
        _check_dtype(mask_targets, torch.int64, "mask_targets")
    _check_dtype(cls_targets, torch.int64, "cls_targets")
    _check_dtype(point_coords, torch.float32, "point_coords")
    B = mask_logits.shape[1]
    if point_coords.dim() != 3 or point_coords.shape[0] != B or point_coords.shape[2] != 2:
        raise RuntimeError("point_coords must be (B,P,2)")


def reference_point_coords(mask_targets: torch.Tensor, num_points: int, background_index=-1,
                           generator=None) -> torch.Tensor:
    """(B,P,2) points drawn as the reference's *_sampling_py functions draw
    them: torch.rand(1,P,2) on the targets' device, once per image that holds
    a non-background GT id, in image order (rows of other images are zero).
    Reads the per-image presence on the host, like the reference."""
    B = mask_targets.shape[0]
    dev = mask_targets.device
    out = torch.zeros((B, num_points, 2), dtype=torch.float32, device=dev)
    if background_index is not None and background_index >= 0:
        has = (mask_targets != background_index).flatten(1).any(1).tolist()
    else:
        has = [True] * B
    for b in range(B):
        if has[b]:
            out[b] = torch.rand((1, num_points, 2), device=dev, generator=generator)[0]
    return out


def pairwise_mask_loss_sampled_forward(mask_logits, mask_targets, cls_logits, cls_targets,
                                       point_coords, smooth=1.0, sigmoid_scale=1.0,
                                       dice_scale=1.0, cls_scale=1.0, background_index=-1,
                                       mask_gamma=0.0, mask_alpha=-1.0, cls_gamma=0.0,
                                       cls_alpha=-1.0, use_softmax_label_loss=False,
                                       align_corners=False) -> torch.Tensor:
    """(3,L,B,Q,GT_out) point-sampled sigmoid-CE, dice and label costs."""
    _check_sampled(mask_logits, mask_targets, cls_logits, cls_targets, point_coords)
    lib = _lib_handle()
    d = _dims(mask_logits, mask_targets, cls_logits, cls_targets)
    p = _params(smooth, sigmoid_scale, dice_scale, cls_scale, background_index, 0.0, 0.05,
                mask_gamma=mask_gamma, mask_alpha=mask_alpha, cls_gamma=cls_gamma,
                cls_alpha=cls_alpha, use_softmax_label_loss=use_softmax_label_loss)
    L, B, Q = mask_logits.shape[:3]
    P = point_coords.shape[1]
    G = lib.ml_gt_out(d.GT_total, p.background_index)
    if G == 0:
        return torch.zeros((L, B, Q, 0), dtype=torch.float32, device=mask_logits.device)
    out = torch.empty((3, L, B, Q, G), dtype=torch.float32, device=mask_logits.device)
    nbytes = lib.ml_sampled_workspace_size(ctypes.byref(d), ctypes.byref(p), P)
    if nbytes == 0:
        raise RuntimeError(lib.ml_last_error().decode() or "invalid shapes")
    ws = _workspace(nbytes, mask_logits.device)
    _lib.check(lib.ml_pairwise_mask_loss_sampled_forward(
        ctypes.byref(d), ctypes.byref(p), P, int(bool(align_corners)), _dtype_code(mask_logits),
        _ptr(mask_logits), _ptr(mask_targets), _ptr(cls_logits), _ptr(cls_targets),
        _ptr(point_coords), _ptr(out), _ptr(ws), ws.numel(), _stream(mask_logits.device)))
    return out


def mask_matching_sampled_ex(mask_logits, mask_targets, cls_logits, cls_targets, point_coords,
                             smooth=1.0, sigmoid_scale=1.0, dice_scale=1.0, cls_scale=1.0,
                             background_index=-1, inf_thresh=1e30, num_masks=-1.0,
                             force_unmatched_class_to_background=False, topk_matches=1,
                             strategy_id=0, mask_gamma=0.0, mask_alpha=-1.0, cls_gamma=0.0,
                             cls_alpha=-1.0, void_class_index=-1, use_softmax_label_loss=False,
                             align_corners=False, *, num_masks_dev=None, want_saved=False,
                             want_costs=False, want_workspace=False):
    """Point-sampled counterpart of mask_matching_ex: returns (pred_to_gt,
    pred_round, layer_means(3,L), saved or None, costs or None) and, with
    want_workspace, the forward workspace (whose sorted points and samples the
    backward can reuse)."""
    check_status()
    _check_sampled(mask_logits, mask_targets, cls_logits, cls_targets, point_coords)
    lib = _lib_handle()
    dev = mask_logits.device
    d = _dims(mask_logits, mask_targets, cls_logits, cls_targets)
    p = _params(smooth, sigmoid_scale, dice_scale, cls_scale, background_index, 0.0, 0.05,
                inf_thresh, num_masks, force_unmatched_class_to_background, False, topk_matches,
                strategy_id, mask_gamma, mask_alpha, cls_gamma, cls_alpha, void_class_index,
                use_softmax_label_loss, True)
    L, B, Q = mask_logits.shape[:3]
    P = point_coords.shape[1]
    G = lib.ml_gt_out(d.GT_total, p.background_index)
    p2g = torch.empty((L, B, Q), dtype=torch.int64, device=dev)
    prd = torch.empty((L, B, Q), dtype=torch.int64, device=dev)
    means = torch.empty((3, L), dtype=torch.float32, device=dev)
    saved = torch.empty((L, B, Q, 4), dtype=torch.float32, device=dev) if want_saved else None
    costs = (torch.empty((3, L, B, Q, G), dtype=torch.float32, device=dev)
             if want_costs and G > 0 else None)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    nbytes = lib.ml_sampled_workspace_size(ctypes.byref(d), ctypes.byref(p), P)
    if nbytes == 0:
        raise RuntimeError(lib.ml_last_error().decode() or "invalid shapes")
    ws = _workspace(nbytes, dev)
    _lib.check(lib.ml_mask_matching_sampled(
        ctypes.byref(d), ctypes.byref(p), P, int(bool(align_corners)), _dtype_code(mask_logits),
        _ptr(mask_logits), _ptr(mask_targets), _ptr(cls_logits), _ptr(cls_targets),
        _ptr(point_coords), _ptr(num_masks_dev), _ptr(p2g), _ptr(prd), _ptr(means), _ptr(costs),
        _ptr(saved), _ptr(status), _ptr(ws), ws.numel(), _stream(dev)))
    _track_status(status)
    if want_workspace:
        return p2g, prd, means, saved, costs, ws
    return p2g, prd, means, saved, costs


def mask_matching_sampled_backward(grad_layer_mask_mean, grad_layer_dice_mean,
                                   grad_layer_cls_mean, mask_logits, mask_targets, cls_logits,
                                   cls_targets, point_coords, pred_to_gt, saved, smooth=1.0,
                                   sigmoid_scale=1.0, dice_scale=1.0, cls_scale=1.0,
                                   background_index=-1, num_masks=-1.0,
                                   force_unmatched_class_to_background=False, mask_gamma=0.0,
                                   mask_alpha=-1.0, cls_gamma=0.0, cls_alpha=-1.0,
                                   void_class_index=-1, use_softmax_label_loss=False,
                                   align_corners=False, *, num_masks_dev=None,
                                   forward_workspace=None):
    """[grad_mask_logits (logits dtype), grad_cls_logits] of the sampled op.
    ``forward_workspace``: the workspace returned by mask_matching_sampled_ex
    for the same inputs (reuses its sorted points and samples)."""
    check_status()
    _check_sampled(mask_logits, mask_targets, cls_logits, cls_targets, point_coords)
    _check_input(saved, "saved")
    lib = _lib_handle()
    dev = mask_logits.device
    d = _dims(mask_logits, mask_targets, cls_logits, cls_targets)
    p = _params(smooth, sigmoid_scale, dice_scale, cls_scale, background_index, 0.0, 0.05, 1e30,
                num_masks, force_unmatched_class_to_background, False, 1, 0, mask_gamma,
                mask_alpha, cls_gamma, cls_alpha, void_class_index, use_softmax_label_loss, True)
    P = point_coords.shape[1]
    dt = _dtype_code(mask_logits)
    gm = torch.empty_like(mask_logits)
    gc = torch.empty_like(cls_logits)
    nbytes = lib.ml_sampled_backward_workspace_size(ctypes.byref(d), ctypes.byref(p), P, dt)
    if nbytes == 0:
        raise RuntimeError(lib.ml_last_error().decode() or "invalid shapes")
    ws = _workspace(nbytes, dev)
    _lib.check(lib.ml_mask_matching_sampled_backward(
        ctypes.byref(d), ctypes.byref(p), P, int(bool(align_corners)), dt,
        _ptr(grad_layer_mask_mean), _ptr(grad_layer_dice_mean), _ptr(grad_layer_cls_mean),
        _ptr(mask_logits), _ptr(mask_targets), _ptr(cls_logits), _ptr(cls_targets),
        _ptr(point_coords), _ptr(pred_to_gt), _ptr(saved), _ptr(num_masks_dev),
        _ptr(forward_workspace), _ptr(gm), _ptr(gc), _ptr(ws), ws.numel(), _stream(dev)))
    return [gm, gc]
