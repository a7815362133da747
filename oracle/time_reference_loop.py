"""Times the reference's own CPU path of the SISO scan (the pure PyTorch loop of
mamba3_ssm/ops.py:160-175, which ssm_scan_siso runs for CPU tensors) beside the fp32 C
restatement oracle/scan_ref.c that bench.py's cpu_baseline and --impl reference arms time,
on the same bounded sample of the long-context workload (one batch row x 64 heads x L
positions, P = 64, D = 128), with the same host threads. Checks that both give the same y
and writes oracle/reference_loop_timing.json.

This is test infrastructure for the CPU baseline, run in the container that holds the
reference source (it imports the reference package from --ref, so it cannot run where the
reference is absent):

    python oracle/time_reference_loop.py [--ref /root/reference] [--L 256]
"""

import argparse
import json
import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default="/root/reference")
    ap.add_argument("--L", type=int, default=256)
    ap.add_argument("--reps", type=int, default=3)
    args = ap.parse_args()
    sys.path.insert(0, ROOT)
    from bench import cpu_sample
    from oracle import cpu_ref
    sys.dont_write_bytecode = True  # nothing is written into the reference's tree
    sys.path.insert(0, args.ref)
    import torch
    from mamba3_ssm.ops import ssm_scan_siso  # the reference package
    threads = cpu_ref.max_threads()
    torch.set_num_threads(threads)
    sample = cpu_sample(args.L)
    t_in = [torch.from_numpy(a) for a in sample]
    ssm_scan_siso(*t_in)  # warm-up
    t0 = time.perf_counter()
    for _ in range(args.reps):
        y_ref = ssm_scan_siso(*t_in)
    ref_s = (time.perf_counter() - t0) / args.reps
    cpu_ref.siso_fwd(*sample, nthreads=threads)
    t0 = time.perf_counter()
    for _ in range(args.reps):
        y_port = cpu_ref.siso_fwd(*sample, nthreads=threads)
    port_s = (time.perf_counter() - t0) / args.reps
    yr = y_ref.numpy().astype(np.float64)
    err = float(np.max(np.abs(y_port - yr)) / np.max(np.abs(yr)))
    out = {
        "sample": f"1 batch row x 64 heads x {args.L} positions (P=64, D=128), fp32, bench.cpu_sample",
        "threads": threads,
        "reference_loop": {"what": "mamba3_ssm/ops.py:160-175 (ssm_scan_siso on CPU tensors)",
                           "s_per_call": ref_s, "tokens_per_s": args.L / ref_s},
        "port": {"what": "oracle/scan_ref.c (OpenMP over (b, h))", "s_per_call": port_s,
                 "tokens_per_s": args.L / port_s},
        "port_over_reference": ref_s / port_s,
        "y_rel_err": err,
    }
    with open(os.path.join(HERE, "reference_loop_timing.json"), "w") as f:
        json.dump(out, f, indent=1)
    print(json.dumps(out, indent=1))


if __name__ == "__main__":
    main()
