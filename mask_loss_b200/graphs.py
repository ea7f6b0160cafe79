"""CUDA-graph capture of a whole matching + loss step.

A training loop with fixed shapes (padded Q, fixed image size and GT slots)
issues the same ~20 launches every step; from Python that costs more host
time than the GPU work at the Mask2Former COCO shape.  ``MatchingLossStep``
captures cost kernels, the on-device solver, the matched-loss forward, the
backward and the optional num_masks all-reduce once, and replays them with one
``cudaGraphLaunch`` per step.

Usage::

    step = MatchingLossStep(mask_logits, mask_targets, cls_logits, cls_targets,
                            *matching_args)      # the 20 scalar args of MaskMatchingFunction
    step.inputs["mask_logits"].copy_(new_logits)  # or write into them in place
    step.replay()
    step.losses          # (3, L): mask, dice, class means
    step.grad_mask_logits, step.grad_cls_logits, step.pred_to_gt, step.pred_round
    step.check()         # raises if a replay's solver reported failure

The inputs are the caller's tensors (kept as static buffers).  ``num_masks``
may be ``"allreduce"``: the per-image GT count is then all-reduced over the
default process group inside the graph (NCCL supports capture).
"""
from __future__ import annotations

import torch

from . import ops, parallel
from .functions.matching import resolve_args
from .functions.sampled import resolve_sampled_args


def _multi_rank() -> bool:
    import torch.distributed as dist
    return dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1


class MatchingLossStep:
    """With ``point_coords`` (B,P,2) the step runs the point-sampled op
    (MaskMatchingSampledFunction) and ``args`` are its 17 scalar arguments;
    otherwise MaskMatchingFunction's 20.  ``zero_fill_beside_solver``: with
    label-map targets, zero the mask gradient on a side stream while the
    solver runs and let the backward write only the rows with a gradient.
    Off by default: measured on B200 the concurrent fill slows the step
    (config 2 in bf16: 0.211 -> 0.242 ms) more than it hides."""

    def __init__(self, mask_logits, mask_targets, cls_logits, cls_targets, *args,
                 point_coords=None, warmup: int = 2, loss_weights=(1.0, 1.0, 1.0),
                 zero_fill_beside_solver: bool = False):
        self.sampled = point_coords is not None
        nargs = 17 if self.sampled else 20
        if len(args) != nargs:
            raise ValueError(f"expected {nargs} scalar arguments after the four tensors")
        self.inputs = {"mask_logits": mask_logits, "mask_targets": mask_targets,
                       "cls_logits": cls_logits, "cls_targets": cls_targets}
        if self.sampled:
            self.inputs["point_coords"] = point_coords
        self.args = list(args)
        self.nm_slot = 6 if self.sampled else 9
        self.allreduce_num_masks = (isinstance(args[self.nm_slot], str) and
                                    args[self.nm_slot] == "allreduce")
        if self.allreduce_num_masks and not _multi_rank():
            # one rank: the count needs no collective, take it from the forward
            self.args[self.nm_slot] = "auto"
            self.allreduce_num_masks = False
        self.w = loss_weights
        self._wts = None
        self._side = None
        self._ev = None
        self._zs = None
        self.prezero = bool(zero_fill_beside_solver)
        self.graph = None
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(max(1, warmup)):  # sets kernel attributes, resolves entry points
                self._run()
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        n0 = len(ops._captured)
        from . import _lib
        l0 = _lib.load().ml_launch_count()
        with torch.cuda.graph(self.graph):
            out = self._run()
        self.kernels_per_replay = int(_lib.load().ml_launch_count() - l0)
        self._flags = ops._captured[n0:]
        del ops._captured[n0:]
        (self.pred_to_gt, self.pred_round, self.losses, self.grad_mask_logits,
         self.grad_cls_logits) = out

    def _run(self):
        """One step through the ops directly (the forward op, then the backward
        op with the loss weights as upstream gradients): the same kernels and
        results as MaskMatchingFunction + autograd, without autograd's glue
        kernels in the graph."""
        ml = self.inputs["mask_logits"]
        mt = self.inputs["mask_targets"]
        cl = self.inputs["cls_logits"]
        ct = self.inputs["cls_targets"]
        for t, n in ((ml, "mask_logits"), (cl, "cls_logits")):
            if not t.is_contiguous():
                raise RuntimeError(f"{n} must be contiguous")
        if cl.dtype != torch.float32:
            raise RuntimeError("cls_logits must be float32")
        a = list(self.args)
        ev = None
        main = torch.cuda.current_stream()
        if self.allreduce_num_masks and not self.sampled:
            # GT count + all-reduce on a side stream: only the forward's matched-loss
            # kernel waits for it, so the collective overlaps costs and solver
            if self._side is None:
                self._side = torch.cuda.Stream(device=ml.device)
                self._ev = torch.cuda.Event()
            self._side.wait_stream(main)
            with torch.cuda.stream(self._side):
                a[self.nm_slot] = parallel.global_num_masks(
                    ops.count_masks(mt, ct.shape[1], int(a[4])))
                self._ev.record(self._side)
            ev = self._ev
        elif self.allreduce_num_masks:
            a[self.nm_slot] = parallel.global_num_masks(ops.count_masks(mt, ct.shape[1], int(a[4])))
        L = ml.shape[0]
        if self._wts is None:
            self._wts = [torch.full((L,), float(w), dtype=torch.float32, device=ml.device)
                         for w in self.w]
        wm, wd, wc = self._wts
        if self.sampled:
            pc = self.inputs["point_coords"]
            args, nm_dev = resolve_sampled_args(*a, device=ml.device)
            p2g, prd, means, saved, _, fws = ops.mask_matching_sampled_ex(
                ml, mt, cl, ct, pc, *args, num_masks_dev=nm_dev, want_saved=True,
                want_workspace=True)
            gm, gc = ops.mask_matching_sampled_backward(
                wm, wd, wc, ml, mt, cl, ct, pc, p2g, saved, args[0], args[1], args[2], args[3],
                args[4], args[6], args[7], args[10], args[11], args[12], args[13], args[14],
                args[15], args[16], num_masks_dev=nm_dev, forward_workspace=fws)
        else:
            dense = ops.is_dense(mt)
            if ml.dtype not in (torch.float32, torch.bfloat16, torch.float16):
                raise RuntimeError("mask_logits must be float32, bfloat16 or float16")
            args, nm_dev = resolve_args(ml, mt, cl, ct, *a)
            # label maps: the mask gradient is zero-filled on a side stream
            # while the solver runs (it needs nothing but the costs' end), and
            # the backward writes only the rows that carry a gradient
            prezero = self.prezero and not dense
            gm_buf = None
            if prezero:
                if self._zs is None:
                    self._zs = torch.cuda.Stream(device=ml.device)
                    self._costs_ev = torch.cuda.Event()
                    self._zero_ev = torch.cuda.Event()
                    # torch creates an event's handle on its first record; the
                    # library records costs_ev itself, so create both now
                    self._costs_ev.record(main)
                    self._zero_ev.record(main)
                gm_buf = torch.empty_like(ml)
            out = ops.mask_matching_ex(
                ml, mt, cl, ct, *args, num_masks_dev=nm_dev, want_saved=True,
                check_void_targets=True, loss_wait_event=ev, want_workspace=not dense,
                costs_done_event=self._costs_ev if prezero else None)
            p2g, prd, means, saved = out[:4]
            fws = None if dense else out[5]
            if prezero:
                self._zs.wait_event(self._costs_ev)
                with torch.cuda.stream(self._zs):
                    gm_buf.zero_()
                    self._zero_ev.record(self._zs)
                gm_buf.record_stream(self._zs)
                main.wait_event(self._zero_ev)
            if ev is not None:
                main.wait_stream(self._side)  # join the side branch
            gm, gc = ops.mask_matching_backward(
                wm, wd, wc, ml, mt, cl, ct, p2g, args[0], args[1], args[2], args[3], args[4],
                args[5], args[6], args[8], args[9], args[10], args[13], args[14], args[15],
                args[16], args[17], args[18], args[19], saved=saved, num_masks_dev=nm_dev,
                forward_workspace=fws, grad_mask_out=gm_buf, grad_rows_prezeroed=prezero)
        return p2g, prd, means, gm, gc

    def replay(self) -> None:
        self.graph.replay()

    def check(self) -> None:
        """Raise if the last replay's solver (or argument check) reported
        failure.  Synchronises."""
        for flag, msg in self._flags:
            v = int(flag.reshape(-1)[0].item())
            if v != 0:
                raise RuntimeError(msg(v) if callable(msg) else msg)
