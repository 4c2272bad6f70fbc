"""Times the NeRF MLP's inference forward on one GPU: the tcgen05 kernel (zf_nerf_mlp_forward_tc through the C ABI)
against the cuBLAS chain of ZipNeRFCudaBackend.NerfMlp, on the reference model's widths (nerf_mlp.cu:440-455) and a
training step's NeRF level (65,536 rays x 32 intervals by default). CUDA events on the current stream, the mean of
--iters runs after 3 warm-ups. Prints one line per implementation.

    python tests/bench_nerf_mlp.py [--samples 2097152] [--iters 10]
"""
from __future__ import annotations

import argparse
import sys
from pathlib import Path

REPO = Path(__file__).resolve().parent.parent
sys.path[:0] = [str(REPO / 'fused-zipnerf_b200')]

import torch  # noqa: E402

MACS_PER_SAMPLE = 64 * 56 + 256 * 96 + 8 * 96 + 2 * 256 * 256 + 8 * 256  # density, combined, skip, view_1, view_2, rgb


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument('--samples', type=int, default=65536 * 32)
    parser.add_argument('--iters', type=int, default=10)
    args = parser.parse_args()
    import ZipNeRFCudaBackend as backend
    from zipnerf_b200 import capi, nerf_mlp as nm
    device = torch.device('cuda')
    layout = nm.NerfMlpLayout()
    gen = torch.Generator().manual_seed(7)
    params = torch.zeros(layout.numel)
    layout.initialize(params, gen)
    n = args.samples
    features = torch.randn(n, 56, generator=gen).bfloat16().to(device)
    inputs = torch.zeros(n, 96, dtype=torch.bfloat16, device=device)
    inputs[:, 64:91] = (torch.rand(n, 27, generator=gen) * 2 - 1).bfloat16().to(device)
    inputs[:, 95] = 1.0
    outputs = torch.empty(n, 8, dtype=torch.bfloat16, device=device)
    status = torch.zeros(1, dtype=torch.int32, device=device)
    packed = {k: v.to(device) for k, v in nm.pack(layout, params).items()}
    mlp = backend.NerfMlp(50, 64, 256, 256, 4)
    flat = mlp.pack(params.to(device))

    def time_ms(fn) -> float:
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(args.iters):
            fn()
        end.record()
        torch.cuda.synchronize()
        return start.elapsed_time(end) / args.iters

    flop = 2 * MACS_PER_SAMPLE * n
    for name, fn in (('tcgen05 zf_nerf_mlp_forward_tc', lambda: capi.nerf_mlp_forward_tc(features, inputs, packed, outputs, status)),
                     ('cuBLAS NerfMlp.forward', lambda: mlp.forward(features, inputs, flat, False))):
        ms = time_ms(fn)
        print(f'{name}: {ms:.3f} ms for {n} samples ({flop / ms / 1e9:.0f} TFLOP/s)', flush=True)
    if int(status.item()) != 0:
        raise SystemExit('a wait of the tensor-core kernel ran out')


if __name__ == '__main__':
    main()
