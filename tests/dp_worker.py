"""One rank of the two-GPU data-parallel test (launched by torchrun from
tests/test_dp_gpu.py): three DataParallel steps over NCCL on a seeded
scene, rank r training view (step * world + r) % 3; saves its parameters.

  torchrun --nproc-per-node 2 tests/dp_worker.py OUT_DIR N WIDTH HEIGHT SEED MODE [VPR]

MODE is the DataParallel mode: "peer" (NVLink kernel) or "nccl".  With
VPR > 1 every step is a batch of world * VPR views, rank r training batch
entries r, r + world, ... (camera (step * world * VPR + entry) % 3).
"""
from __future__ import annotations

import math
import os
import sys

import numpy as np
import torch

from msplat_b200 import engine, multigpu, synthetic
from tests import harness


def main():
    out_dir, n, w, h, seed = sys.argv[1], *map(int, sys.argv[2:6])
    mode = sys.argv[6]
    vpr = int(sys.argv[7]) if len(sys.argv) > 7 else 1
    rank, world = multigpu.rank_and_world()
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
    engine.bind_stream()
    g = synthetic.gaussians(n, seed, mean_range=1.0, log_scale_mu=math.log(0.02),
                            log_scale_sigma=0.3)
    cams = [synthetic.front_camera(w, h, 3.0 + 0.3 * k) for k in range(3)]
    model = engine.GaussianModel(g.groups())
    dp = multigpu.DataParallel(model, rank, world, timeout_s=60, mode=mode, views_per_rank=vpr)
    for step in range(3):
        css, gts = [], []
        for k in range(vpr):
            v = (step * world * vpr + k * world + rank) % 3
            cs = harness.setup_cam(cams[v])
            gen = torch.Generator(device="cuda").manual_seed(v)
            css.append(cs)
            gts.append(torch.rand(cs.height, cs.width, 3, device="cuda", generator=gen))
        dp.train_views(css, gts)
    torch.cuda.synchronize()
    dp.barrier()
    if mode == "peer":
        assert dp.peer_errors() == 0, "peer step timed out"
    np.savez(os.path.join(out_dir, f"rank{rank}.npz"),
             **{f"p{i}": model.params[i].cpu().numpy() for i in range(6)})
    dp.shutdown()


if __name__ == "__main__":
    main()
