"""World-size-2 data parallelism on CPU (gloo): the sharding and the two
collectives of mask_loss_b200.parallel reproduce the single-process result.
The per-rank compute is the CPU oracle (the GPU kernels are covered by the
-m gpu tests); this checks the host-side logic that bench.py uses."""
import os

import numpy as np
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from mask_loss_b200 import parallel, synthetic
from oracle import oracle as O

CFG = synthetic.Config("dp", 11, 1, 4, 12, 16, 16, 1, 7, 3.0, "ellipse", ("fixed", 4), (0.02, 0.2))


def _kw():
    kw = synthetic.parity_kwargs(CFG)
    return kw


def _rank_losses(images, num_masks):
    b = synthetic.make_batch(CFG, images=images)
    P = O.Params(**{**_kw(), "num_masks": float(num_masks)})
    x, t, z, y = (b[k].numpy() for k in ("mask_logits", "mask_targets", "cls_logits", "cls_targets"))
    _, _, m, d, c, _ = O.mask_matching(x, t, z, y, P)
    gt = int(sum((np.unique(t[i]) > 0).sum() for i in range(len(images))))
    return np.array([m[0], d[0], c[0]]), gt


def _worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    imgs = list(parallel.shard_images(CFG.B, rank, world))
    _, gt = _rank_losses(imgs, 1.0)
    nm = parallel.global_num_masks(torch.tensor(float(gt)))
    losses, _ = _rank_losses(imgs, float(nm))
    lt = torch.tensor(losses)
    parallel.average_losses(lt)
    if rank == 0:
        out.put((float(nm), lt.numpy()))
    dist.barrier()
    dist.destroy_process_group()


def test_two_rank_gloo_matches_single_process():
    import socket
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    nm, got = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    # single process over all images, num_masks = total GT count
    _, gt_all = _rank_losses(list(range(CFG.B)), 1.0)
    ref, _ = _rank_losses(list(range(CFG.B)), float(gt_all))
    assert abs(nm * 2 - gt_all) < 1e-6
    # mask/dice: normalised by the global count -> identical; the forced class
    # term uses the per-shard B*Q, whose mean over equal shards is identical too
    np.testing.assert_allclose(got, ref, rtol=1e-6)


def test_shards_cover_batch():
    for B, W in [(16, 8), (7, 3), (64, 4)]:
        seen = [i for r in range(W) for i in parallel.shard_images(B, r, W)]
        assert seen == list(range(B))
