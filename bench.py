"""Benchmark: images/s of Mask2Former-style matching + loss, forward + backward.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config cfg2] [--impl ours|reference]
                    [--logits fp32|bf16|fp16] [--targets labels|dense]

One step = one pass of the hot path over one batch: pairwise costs, on-device
assignment, matched losses (forward) and dL/dlogits (backward) through
``mask_loss_b200.functions.MaskMatchingFunction``.  Workload: the
Mask2Former COCO-panoptic shape (config 2: B=16 images per GPU, Q=100,
256x256 fp32 logits, label maps with Poisson(15) GTs, C'=134), seeded
synthetic data.  Inputs (419 MB of logits per GPU) are larger than the L2, so
no flush is needed between steps.

N > 1: launched by torchrun, one rank per GPU, weak scaling (16 images per
GPU); the only collectives are an NCCL all-reduce of num_masks (before the
loss) and of the loss scalars (reporting).  Timing is device-side (CUDA
events), max over ranks.

Other workloads: --config cfg1/cfg3/cfg4/cfg5/native (the configs of
mask_loss_b200/synthetic.py; native = the reference harness's own shape, 8 x
Q=128 x 256^2 logits against 1024^2 label maps), --logits bf16/fp16 (16-bit
mask logits, widened in the kernels), --targets dense (per-GT uint8 masks cut
from the label maps, one GPU).  The default line is config 2, fp32.

--impl reference times the CPU implementation of the same path on the host
cores: the CPU restatement in oracle/ for costs and losses, and the
reference's own compiled C++ solver (oracle/_ref) when it was built.  Under
torchrun only rank 0 runs it.

Prints one JSON line on rank 0.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import tempfile
import time

import numpy as np
import torch

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

METRIC = "images/sec matching+loss fwd+bwd (Mask2Former shape)"
UNIT = "images/s"


_JSON_FD = None  # the original stdout when library chatter is moved to stderr


def emit(line: dict) -> None:
    """Print the one JSON result line on the real stdout."""
    text = json.dumps(line) + "\n"
    if _JSON_FD is None:
        sys.stdout.write(text)
        sys.stdout.flush()
    else:
        os.write(_JSON_FD, text.encode())


def quiet_stdout() -> None:
    """Send everything else written to fd 1 (NCCL's version banner, library
    logs) to stderr, so stdout carries only the JSON line."""
    global _JSON_FD
    if _JSON_FD is None:
        sys.stdout.flush()
        _JSON_FD = os.dup(1)
        os.dup2(2, 1)


def dist_info():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


# ---------------------------------------------------------------------------
# clocks during the timed region
# ---------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None
        self.path = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            self.fh = os.fdopen(fd, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "20", "-i", str(self.idx)],
                stdout=self.fh, stderr=subprocess.DEVNULL)
            time.sleep(0.3)  # let the sampler come up before the timed region
        except (OSError, FileNotFoundError):
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.fh.close()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        try:
            for line in open(self.path):
                f = [x.strip() for x in line.split(",")]
                if len(f) < 9:
                    continue
                try:
                    sm.append(float(f[1]))
                    mx = float(f[2])
                except ValueError:
                    continue
                for n, v in zip(names, f[5:9]):
                    if v.lower().startswith("active"):
                        reasons.add(n)
        finally:
            os.unlink(self.path)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------------------
# CPU implementation (oracle port + reference solver), images/s
# ---------------------------------------------------------------------------
def cpu_images_per_sec(cfg, n_images: int, threads: int, start: int = 0):
    """Run the CPU path on `n_images` images (one image per task) with
    `threads` host threads; returns (images/s, seconds, solver kind)."""
    from concurrent.futures import ThreadPoolExecutor

    from mask_loss_b200 import synthetic
    from oracle import oracle as O

    O.lib()
    use_ref = O.ref_lib() is not None
    kw = synthetic.parity_kwargs(cfg)
    P = O.Params(**kw)
    idx = [(start + i) % cfg.B for i in range(n_images)]
    batches = [synthetic.make_batch(cfg, images=[b]) for b in idx]
    for bt in batches:
        bt["mask_logits"] = bt["mask_logits"].numpy()
        bt["cls_logits"] = bt["cls_logits"].numpy()
        bt["mask_targets"] = bt["mask_targets"].numpy()
        bt["cls_targets"] = bt["cls_targets"].numpy()

    def one(bt):
        x, t, z, y = bt["mask_logits"], bt["mask_targets"], bt["cls_logits"], bt["cls_targets"]
        p2g, prd, m, d, c, _ = O.mask_matching(x, t, z, y, P, use_ref=use_ref)
        O.mask_matching_backward([1.0] * cfg.L, [1.0] * cfg.L, [1.0] * cfg.L, x, t, z, y, p2g, P)
        return float(m[0] + d[0] + c[0])

    t0 = time.perf_counter()
    with ThreadPoolExecutor(max_workers=threads) as ex:
        list(ex.map(one, batches))
    dt = time.perf_counter() - t0
    return n_images / dt, dt, ("reference C++ solver (oracle/_ref)" if use_ref else "C restatement")


def run_reference(args, cfg):
    ws, rank, _ = dist_info()
    if rank != 0:
        return
    threads = max(1, os.cpu_count() or 1)
    per_step = min(threads, 2 * cfg.B)
    for w in range(max(0, min(args.warmup, 1))):
        cpu_images_per_sec(cfg, min(per_step, threads), threads)
    times = []
    solver = ""
    budget_s = float(os.environ.get("MASK_LOSS_B200_REF_BUDGET_S", "120"))
    for k in range(args.steps):
        _, dt, solver = cpu_images_per_sec(cfg, per_step, threads, start=k * per_step)
        times.append(dt)
        if sum(times) > budget_s:  # bounded: stop early, report the steps run
            break
    done = len(times)
    total = sum(times)
    value = per_step * done / total
    sample = (f"{per_step} images of {cfg.name} per step ({cfg.B}-image batch shape), one image per "
              f"host thread; costs/losses/grads by the C restatement in oracle/, assignment by "
              f"the {solver}")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": ws,
        "steps": done, "steps_requested": args.steps, "warmup": args.warmup,
        "ms_per_step": 1e3 * total / done,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": f"synthetic (seeded, {cfg.name} shapes)",
        "config": {"workload": cfg.name, "images_per_step": per_step, "Q": cfg.Q,
                   "HW": f"{cfg.H}x{cfg.W}", "classes": cfg.C},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    emit(line)


# ---------------------------------------------------------------------------
# GPU implementation
# ---------------------------------------------------------------------------
def read_traffic(cfg_name: str, kernel: str = "cost_partial_kernel"):
    """DRAM bytes per launch of the cost kernel from the committed ncu summary."""
    p = os.path.join(REPO, "profiles", f"{kernel}_{cfg_name}.md")
    try:
        for line in open(p):
            if line.startswith("traffic_bytes_per_launch:"):
                return float(line.split(":")[1])
    except OSError:
        pass
    return None


def run_ours(args, cfg):
    import torch.distributed as dist

    from mask_loss_b200 import _lib, ops, parallel, synthetic
    from mask_loss_b200 import functions as F

    ws, rank, local = dist_info()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if ws > 1:
        dist.init_process_group("nccl", device_id=dev)
    lib = _lib.load()

    # this rank's shard: images [rank*B, (rank+1)*B) of the global batch
    imgs = list(parallel.shard_images(ws * cfg.B, rank, ws))
    batch = synthetic.make_batch(cfg, images=imgs, device="cpu", logits=False)
    mt = batch["mask_targets"].to(dev)
    ct = batch["cls_targets"].to(dev)
    g = torch.Generator(device=dev).manual_seed(1000 * cfg.cfg + 7 + rank)
    ml = torch.randn((cfg.L, cfg.B, cfg.Q, cfg.H, cfg.W), generator=g, device=dev) * cfg.logit_std
    cl = torch.randn((cfg.L, cfg.B, cfg.Q, cfg.C), generator=g, device=dev)
    kw = synthetic.parity_kwargs(cfg)
    GT_total = ct.shape[1]
    sampled = cfg.name == "cfg3"
    dense = args.targets == "dense"
    if dense:
        # per-GT masks (B, GT_total, Ht, Wt) uint8 cut from the label maps
        if ws > 1 or sampled:
            raise SystemExit("--targets dense runs on one GPU with a label-map config")
        mt = torch.stack([mt == g for g in range(GT_total)], 1).to(torch.uint8).contiguous()
    pc = None
    half = {"bf16": torch.bfloat16, "fp16": torch.float16}.get(args.logits)
    if half is not None and not sampled:
        # 16-bit mask logits end to end (the kernels widen them; the gradient
        # is written in the same type)
        ml = ml.to(half)
    if sampled:  # point-sampled configuration: bf16 logits, P points per image
        ml = ml.to(torch.bfloat16)
        gp = torch.Generator(device=dev).manual_seed(31 + rank)
        pc = torch.rand((cfg.B, synthetic.CFG3_POINTS, 2), generator=gp, device=dev)

    def sargs(nm):
        return (kw["smooth"], kw["sigmoid_scale"], kw["dice_scale"], kw["cls_scale"],
                kw["background_index"], kw["inf_thresh"], nm, True, 1, "global", 0.0, None, None,
                None, kw["void_class_index"], "softmax", False)

    def step(ml_in, mt_in, cl_in, ct_in):
        if dense:
            nm = "auto"  # the forward counts the non-empty masks itself
        else:
            nm = parallel.global_num_masks(ops.count_masks(mt_in, ct_in.shape[1],
                                                           kw["background_index"]))
        x = ml_in.detach().requires_grad_(True)
        z = cl_in.detach().requires_grad_(True)
        if sampled:
            p2g, prd, m, d, c = F.MaskMatchingSampledFunction.apply(x, mt_in, z, ct_in, pc,
                                                                    *sargs(nm))
        else:
            p2g, prd, m, d, c = F.MaskMatchingFunction.apply(
                x, mt_in, z, ct_in, kw["smooth"], kw["sigmoid_scale"], kw["dice_scale"],
                kw["cls_scale"], kw["background_index"], kw["uncertainty_gamma"],
                kw["uncertainty_gamma_min"], True, kw["inf_thresh"], nm, True, False, 1, "global",
                0.0, None, None, None, kw["void_class_index"], "softmax")
        losses = torch.stack([m, d, c])
        losses.sum().backward()
        losses = losses.detach()
        parallel.average_losses(losses, async_op=True)
        return losses, x.grad, z.grad, p2g

    def barrier():
        torch.cuda.synchronize()
        if ws > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def timed(fn, n):
        barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(n):
            fn()
        e1.record()
        barrier()
        ms = e0.elapsed_time(e1)
        if ws > 1:
            t = torch.tensor([ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms

    for _ in range(args.warmup):
        step(ml, mt, cl, ct)
    # ---- eager steps with the library's per-kernel event hooks (stage times) ----
    lib.ml_profile_enable(1)
    n_eager = max(3, min(args.steps, 50))
    ms_eager = timed(lambda: step(ml, mt, cl, ct), n_eager) / n_eager
    lib.ml_profile_enable(0)
    NK = 7  # profile kinds of the library (include/mask_loss_b200.h, ml_profile_enable)
    kms = np.zeros(NK, np.float32)
    kn = np.zeros(NK, np.int64)
    lib.ml_profile_read(kms.ctypes.data, kn.ctypes.data, NK)
    kstep = kms / n_eager  # ms per step of each kind
    # matched query rows of one step (the gradient stage re-reads their logits)
    matched = int((step(ml, mt, cl, ct)[3] >= 0).sum().item()) if not sampled else None

    # ---- device-resident throughput (value): the whole step as one CUDA graph ----
    from mask_loss_b200.graphs import MatchingLossStep
    g_ml, g_mt, g_cl, g_ct = ml.clone(), mt.clone(), cl.clone(), ct.clone()
    if sampled:
        gstep = MatchingLossStep(g_ml, g_mt, g_cl, g_ct, *sargs("allreduce"), point_coords=pc,
                                 warmup=max(1, args.warmup))
    else:
        gstep = MatchingLossStep(
            g_ml, g_mt, g_cl, g_ct, kw["smooth"], kw["sigmoid_scale"], kw["dice_scale"],
            kw["cls_scale"], kw["background_index"], kw["uncertainty_gamma"],
            kw["uncertainty_gamma_min"], True, kw["inf_thresh"], "allreduce", True, False, 1,
            "global", 0.0, None, None, None, kw["void_class_index"], "softmax",
            warmup=max(1, args.warmup))
    for _ in range(args.warmup):
        gstep.replay()
    # stage A alone (label codes, cost kernel, finalize) as its own graph
    ms_stage_a = None
    if not sampled:
        a_out = {}

        def stage_a():
            a_out["c"] = ops.pairwise_mask_loss_forward(
                g_ml, g_mt, g_cl, g_ct, kw["smooth"], kw["sigmoid_scale"], kw["dice_scale"],
                kw["cls_scale"], kw["background_index"], kw["uncertainty_gamma"],
                kw["uncertainty_gamma_min"], 0.0, -1.0, 0.0, -1.0, True, True)

        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            stage_a()
        torch.cuda.current_stream().wait_stream(side)
        ga = torch.cuda.CUDAGraph()
        with torch.cuda.graph(ga):
            stage_a()
        for _ in range(args.warmup):
            ga.replay()
        ms_stage_a = timed(ga.replay, args.steps) / args.steps
        ga = None
    # the same step with the gradient zero fill beside the solver (for comparison)
    ms_noprezero = None
    if not sampled and not dense:
        nstep = MatchingLossStep(
            g_ml, g_mt, g_cl, g_ct, kw["smooth"], kw["sigmoid_scale"], kw["dice_scale"],
            kw["cls_scale"], kw["background_index"], kw["uncertainty_gamma"],
            kw["uncertainty_gamma_min"], True, kw["inf_thresh"], "allreduce", True, False, 1,
            "global", 0.0, None, None, None, kw["void_class_index"], "softmax",
            warmup=max(1, args.warmup), zero_fill_beside_solver=True)
        for _ in range(args.warmup):
            nstep.replay()
        ms_noprezero = timed(nstep.replay, args.steps) / args.steps
        nstep = None
    # the reference's user-facing call: MaskMatchingFunction.apply + backward()
    ms_eager_fn = None
    if not sampled:
        def eager_fn():
            x = ml.detach().requires_grad_(True)
            z = cl.detach().requires_grad_(True)
            _, _, m, d, c = F.MaskMatchingFunction.apply(
                x, mt, z, ct, kw["smooth"], kw["sigmoid_scale"], kw["dice_scale"],
                kw["cls_scale"], kw["background_index"], kw["uncertainty_gamma"],
                kw["uncertainty_gamma_min"], True, kw["inf_thresh"], None, True, False, 1,
                "global", 0.0, None, None, None, kw["void_class_index"], "softmax")
            (m + d + c).backward()

        for _ in range(args.warmup):
            eager_fn()
        n_fn = max(3, min(args.steps, 50))
        ms_eager_fn = timed(eager_fn, n_fn) / n_fn
    # inputs smaller than the 126 MB L2 (config 3): flush L2 between steps by
    # writing a 256 MB buffer, and subtract the flush time measured alone
    in_bytes = sum(t.numel() * t.element_size() for t in (g_ml, g_mt, g_cl, g_ct))
    flush_ms = 0.0
    step_fn = gstep.replay
    if in_bytes < 160 << 20:
        flush_buf = torch.empty(64 << 20, dtype=torch.float32, device=dev)

        def step_fn():
            flush_buf.zero_()
            gstep.replay()

        flush_ms = timed(flush_buf.zero_, args.steps) / args.steps
    clocks = ClockSampler(local)
    clocks.start()
    ms = timed(step_fn, args.steps) - flush_ms * args.steps
    clk = clocks.stop()
    gstep.check()
    launches = gstep.kernels_per_replay * args.steps
    ms_step = ms / args.steps
    value = ws * cfg.B * cfg.L / (ms_step / 1e3)

    # ---- end to end through the public API with host buffers ----
    h_ml = ml.cpu().pin_memory()
    h_mt = mt.cpu().pin_memory()
    h_cl = cl.cpu().pin_memory()
    h_ct = ct.cpu().pin_memory()
    h_out = torch.empty((3, cfg.L), dtype=torch.float32).pin_memory()
    h2d = sum(t.numel() * t.element_size() for t in (h_ml, h_mt, h_cl, h_ct))
    d2h = h_out.numel() * h_out.element_size()

    def e2e_step():
        g_ml.copy_(h_ml, non_blocking=True)
        g_mt.copy_(h_mt, non_blocking=True)
        g_cl.copy_(h_cl, non_blocking=True)
        g_ct.copy_(h_ct, non_blocking=True)
        gstep.replay()
        h_out.copy_(gstep.losses, non_blocking=True)

    for _ in range(max(1, args.warmup // 2)):
        e2e_step()
    e2e_steps = max(3, min(args.steps, 20))
    ms_e2e = timed(e2e_step, e2e_steps) / e2e_steps
    e2e = ws * cfg.B * cfg.L / (ms_e2e / 1e3)
    # the same with both logit gradients copied back to pinned host buffers
    h_gm = torch.empty(gstep.grad_mask_logits.shape, dtype=gstep.grad_mask_logits.dtype,
                       pin_memory=True)
    h_gc = torch.empty(gstep.grad_cls_logits.shape, dtype=torch.float32, pin_memory=True)

    def e2e_grads_step():
        e2e_step()
        h_gm.copy_(gstep.grad_mask_logits, non_blocking=True)
        h_gc.copy_(gstep.grad_cls_logits, non_blocking=True)

    e2e_grads_step()
    ms_e2e_g = timed(e2e_grads_step, e2e_steps) / e2e_steps
    d2h_g = d2h + sum(t.numel() * t.element_size() for t in (h_gm, h_gc))
    gstep.check()

    # ---- N > 1: what the num_masks collective costs the step ----
    scaling = None
    if ws > 1 and not sampled:
        # the same graph step with the local GT count (no collective)
        lstep = MatchingLossStep(
            g_ml, g_mt, g_cl, g_ct, kw["smooth"], kw["sigmoid_scale"], kw["dice_scale"],
            kw["cls_scale"], kw["background_index"], kw["uncertainty_gamma"],
            kw["uncertainty_gamma_min"], True, kw["inf_thresh"], "auto", True, False, 1,
            "global", 0.0, None, None, None, kw["void_class_index"], "softmax",
            warmup=max(1, args.warmup))
        for _ in range(args.warmup):
            lstep.replay()
        ms_local = timed(lstep.replay, args.steps) / args.steps
        lstep = None
        # the 4-byte all-reduce alone, back to back
        one = torch.ones(1, device=dev)
        for _ in range(args.warmup):
            dist.all_reduce(one)
        ms_ar = timed(lambda: dist.all_reduce(one), args.steps) / args.steps
        scaling = {"step_ms_allreduce_num_masks": ms_step, "step_ms_local_num_masks": ms_local,
                   "allreduce_4B_us": 1e3 * ms_ar,
                   "note": "max over ranks; local = the same graph step without the collective"}
    ops.check_status(block=True)

    def teardown():
        """All ranks: free the captured graph (it holds NCCL work), barrier,
        destroy the group.  A watchdog force-exits if teardown stalls, so a
        finished benchmark never holds its GPUs."""
        nonlocal gstep
        gstep = None
        torch.cuda.synchronize()
        if ws > 1:
            import threading
            threading.Timer(60.0, lambda: os._exit(0)).start()
            dist.barrier()
            dist.destroy_process_group()
            sys.stdout.flush()
            os._exit(0)

    if rank != 0:
        teardown()
        return
    peaks = {}
    try:
        peaks = json.load(open(os.path.join(REPO, "MEASURED_PEAKS.json")))
    except (OSError, ValueError):
        pass
    peak = peaks.get("hbm_gbs")
    peak_src = "measured" if peak else "fallback"
    peak = peak or 6650.0
    # roofline of the dominant kernel: the streaming cost kernel reads every
    # logit once plus one int32 code per cell and image
    cells = synthetic.CFG3_POINTS if sampled else cfg.H * cfg.W  # sampled values are fp32
    # dense targets run on the tensor-core kernels unless MASK_LOSS_B200_DENSE_MMA=0
    # (the bench's settings have no entropy weights or focal terms, GT_out <= 64):
    # fp32 logits with GT_total <= 64 on the kind::tf32 one (unless
    # MASK_LOSS_B200_DENSE_TF32=0), else the bf16 one (bf16 counts)
    count_bytes = 2
    if os.environ.get("MASK_LOSS_B200_DENSE_MMA", "1")[:1] == "0":
        dense_kernel = "dense_cost_kernel"
    elif (half is None and (GT_total + 15) // 16 * 16 <= 64 and
          os.environ.get("MASK_LOSS_B200_DENSE_TF32", "1")[:1] != "0"):
        # unscaled masks (16-cell rows) are its B source directly: one byte a
        # cell and GT; else fp32 counts
        dense_kernel = "dense_mma_tf32_kernel"
        count_bytes = 1 if (cfg.s == 1 and (cfg.H * cfg.W) % 16 == 0) else 4
    else:
        dense_kernel = "dense_mma_kernel"
        # bf16 logits with unscaled masks: the masks are its B source too
        if half is torch.bfloat16 and cfg.s == 1 and (cfg.H * cfg.W) % 16 == 0:
            count_bytes = 1
    cost_kernel = dense_kernel if dense else "cost_partial_kernel"
    # dense: every logit plus each GT's count per cell
    esize = 2 if (half is not None and not sampled) else 4
    cost_bytes = (cfg.L * cfg.B * cfg.Q * cells * esize +
                  (cfg.B * cells * (GT_total - 1) * count_bytes if dense else cfg.B * cells * 4))
    cost_ms = float(kms[0] / max(kn[0], 1))
    achieved = cost_bytes / (cost_ms / 1e3) / 1e9
    traffic = read_traffic(cfg.name, cost_kernel)
    grad_ms = float(kms[1] / max(kn[1], 1))
    match_ms = float(kms[2] / max(kn[2], 1))
    # stage roofline (per step, algorithmic bytes):
    #   A (costs)   = label map + every logit once + class logits
    #   C (losses)  = the gradient written + the matched rows' logits re-read
    #                 + label map + class logits read and their gradient written
    LBQ = cfg.L * cfg.B * cfg.Q
    lab_bytes = cfg.B * (cfg.H * cfg.s) * (cfg.W * cfg.s) * (GT_total if dense else 8)
    cls_bytes = LBQ * cfg.C * 4
    stages = None
    if not sampled:
        HW = cfg.H * cfg.W
        bytes_a = lab_bytes + LBQ * HW * esize + cls_bytes
        bytes_c = LBQ * HW * esize + matched * HW * esize + lab_bytes + 2 * cls_bytes
        ms_a = float(ms_stage_a)
        ms_b = float(kstep[2])
        ms_c = max(ms_step - ms_a - ms_b, 1e-6)
        stages = {
            "A_costs": {"ms": ms_a, "bytes": bytes_a, "frac": bytes_a / (ms_a / 1e3) / 1e9 / peak,
                        "kernels": f"label_code + {cost_kernel} + cost_rows + "
                                   "cost_pairs, timed as their own CUDA graph"},
            "B_solver": {"ms": ms_b, "kernels": "match_kernel, event-timed (latency-bound, "
                                                "no roofline)"},
            "C_losses_grads": {"ms": ms_c, "bytes": bytes_c,
                               "frac": bytes_c / (ms_c / 1e3) / 1e9 / peak,
                               "kernels": "loss_fwd + bwd_cls + mask_grad; "
                                          "time = step - A - B"},
            "step": {"ms": ms_step, "bytes": bytes_a + bytes_c,
                     "frac": (bytes_a + bytes_c) / (ms_step / 1e3) / 1e9 / peak,
                     "note": "graph-replayed step; bytes of stages A and C"},
            "matched_rows_per_step": matched,
            "event_ms_per_kind": {n: float(kstep[i]) for i, n in enumerate(
                ["cost", "mask_grad", "solver", "label_prep", "cost_finalize", "loss_fwd",
                 "cls_bwd"])},
            "step_ms_with_zero_fill_beside_solver": ms_noprezero,
        }
    cpu = None
    if ws == 1 and not sampled and not dense:
        threads = max(1, os.cpu_count() or 1)
        n_img = min(threads, 2 * cfg.B)
        v, dt, solver = cpu_images_per_sec(cfg, n_img, threads)
        cpu = {"value": v, "unit": UNIT, "cores": threads, "kind": "port",
               "sample": f"{n_img} images of {cfg.name} (one per host thread, {dt:.1f} s); "
                         f"costs/losses/grads by the C restatement in oracle/, assignment by the "
                         f"{solver}"}
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": ws, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None,
        "dtype": ("bf16 logits, f32 math" if sampled else
                  f"{args.logits} logits, f32 math" if half is not None else "f32"),
        "data": (f"synthetic (seeded, {cfg.name} shapes)" +
                 (f"; {synthetic.CFG3_POINTS} uniform points per image" if sampled else
                  "; inputs > L2, no flush needed")),
        "config": {"workload": cfg.name + ("-dense" if dense else "") +
                               (f"-{args.logits}" if half is not None and not sampled else ""),
                   "targets": ("per-GT uint8 masks (B,GT,Ht,Wt)" if dense else "label map (B,Ht,Wt)"),
                   "images_per_gpu": cfg.B, "global_batch": ws * cfg.B,
                   "Q": cfg.Q, "HW": f"{cfg.H}x{cfg.W}", "classes": cfg.C, "K": 1,
                   "strategy": "global", "label_loss": "softmax", "parallelism": f"dp{ws}",
                   "l2": ("inputs larger than L2" if not flush_ms else
                          f"L2 flushed before every step (256 MB write, {flush_ms:.3f} ms, subtracted)")},
        "e2e": {"value": e2e, "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "ms_per_step": ms_e2e,
                "note": "headline: inputs from pinned host memory, loss means back; the "
                        "gradients stay on the device, where the model's backward reads them"},
        "e2e_with_grads": {"value": ws * cfg.B * cfg.L / (ms_e2e_g / 1e3), "unit": UNIT,
                           "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h_g,
                           "ms_per_step": ms_e2e_g,
                           "note": "as e2e, plus both logit gradients copied to pinned host memory"},
        "roofline": {"bound": "hbm", "kernel": cost_kernel, "achieved": achieved,
                     "peak": peak, "unit": "GB/s", "frac": achieved / peak, "traffic": traffic,
                     "algorithmic_bytes_per_launch": cost_bytes, "avg_launch_ms": cost_ms,
                     "peak_source": peak_src},
        "stages_ms": {cost_kernel: cost_ms, "mask_grad_kernel": grad_ms,
                      "match_kernel": match_ms, "eager_step": ms_eager,
                      "eager_fn_ms": ms_eager_fn},
        "stages": stages,
        "multi_gpu": scaling,
        "execution": "value and e2e replay the step as one CUDA graph "
                     "(mask_loss_b200.graphs.MatchingLossStep); stage times from eager steps",
        "gpu_launches": int(launches),
        "clocks": clk,
        "cpu_baseline": cpu,
    }
    emit(line)
    teardown()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", default="cfg2")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--logits", default="fp32", choices=["fp32", "bf16", "fp16"],
                    help="mask-logit type of the label-map configs (cfg3 is always bf16)")
    ap.add_argument("--targets", default="labels", choices=["labels", "dense"],
                    help="dense: per-GT uint8 masks instead of the label map (one GPU)")
    args = ap.parse_args()
    if int(os.environ.get("WORLD_SIZE", "1")) > 1:
        quiet_stdout()
    if args.warmup < 3 and args.impl == "ours":
        args.warmup = 3
    from mask_loss_b200 import synthetic
    cfg = synthetic.CONFIGS[args.config]
    if args.impl == "reference":
        run_reference(args, cfg)
    else:
        run_ours(args, cfg)


if __name__ == "__main__":
    main()
