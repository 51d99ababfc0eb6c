"""Run one workload's forward pass a few times on the device, for profilers.

    python -m forgetune_b200.profile_run --workload residual_mlp --batch 1024 --iters 3

Builds the workload (forgetune_b200.workloads) through the same graph blob
compile_model embeds, generates its input on the device (the counter-based
normal generator, seed 1), runs `--warmup` untimed and `--iters` forward
passes as CUDA-graph replays on one GPU, and prints the per-launch-list-step
device times of one profiled pass.  Meant as the program an ncu capture
wraps: it holds only the workload's weights, input, output and arena on the
device, and launches few kernels before the ones of interest.
"""

from __future__ import annotations

import argparse
import json
import sys

import numpy as np


def main(argv=None) -> int:
    import torch

    from forgetune_b200 import _native, workloads
    from forgetune_b200.frontend import export_to_ir
    from forgetune_b200.graph_blob import serialize

    ap = argparse.ArgumentParser()
    ap.add_argument("--workload", required=True, choices=sorted(workloads.WORKLOADS))
    ap.add_argument("--batch", type=int, required=True)
    ap.add_argument("--iters", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=1)
    ap.add_argument("--policy", default="auto", choices=["auto", "simt", "simt_exact", "tcgen05"])
    ap.add_argument("--tile", default=None,
                    help="tc_bn,tc_bk,tc_mh,tc_pair for every GEMM step (ftb_model_set_step_config), e.g. 128,32,0,3")
    args = ap.parse_args(argv)

    builder, shape, _ = workloads.WORKLOADS[args.workload]
    model = builder()
    B = args.batch
    ir = export_to_ir(model, (torch.zeros((2,) + tuple(shape)),), dynamic_batch=True, max_batch_size=max(B, 2))
    eng = _native.EngineModel(serialize(ir, enable_fusion=True, bias_first_fused=True, kernel_policy=args.policy))
    dev = torch.cuda.current_device()
    eng.set_devices([dev])
    if args.tile:
        bn, bk, mh, pair = (int(v) for v in args.tile.split(","))
        for i, st in enumerate(eng.desc["steps"]):
            if st.get("kind") == 0:
                eng.set_step_config(i, bn, bk, mh, pair, True)
    eng.prepare()
    n_in = B * int(np.prod(shape))
    with torch.no_grad():
        out_f = int(model(torch.zeros((1,) + tuple(shape))).shape[1])
    x = torch.empty(n_in, dtype=torch.float32, device="cuda")
    y = torch.empty(B * out_f, dtype=torch.float32, device="cuda")
    stream = torch.cuda.current_stream()
    _native.philox_normal(x.data_ptr(), 1, 0, n_in, stream.cuda_stream)
    for _ in range(args.warmup):
        eng.run_device(x.data_ptr(), n_in, y.data_ptr(), B * out_f, B, stream.cuda_stream)
    for _ in range(args.iters):
        eng.run_device(x.data_ptr(), n_in, y.data_ptr(), B * out_f, B, stream.cuda_stream)
    ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
    ev[0].record(stream)
    for _ in range(args.iters):
        eng.run_device(x.data_ptr(), n_in, y.data_ptr(), B * out_f, B, stream.cuda_stream)
    ev[1].record(stream)
    eng.run_device_profiled(x.data_ptr(), n_in, y.data_ptr(), B * out_f, B, stream.cuda_stream, 0)
    torch.cuda.synchronize()
    warm_ms = ev[0].elapsed_time(ev[1]) / max(1, args.iters)
    steps = eng.desc["steps"]
    per_step = eng.profile_read(0)
    print(json.dumps({"workload": args.workload, "batch": B, "kernels_per_forward": eng.graph_kernels(),
                      "ms_per_forward_l2_warm": round(warm_ms, 5), "tile": args.tile,
                      "steps": [{"kind": s.get("kind"), "K": s.get("K"), "N": s.get("N"), "ms": round(t, 5)}
                                for s, t in zip(steps, per_step)]}))
    eng.close()
    return 0


if __name__ == "__main__":
    sys.exit(main())
