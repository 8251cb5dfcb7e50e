"""Golden vectors of the rotated quantizer, made by the reference's own rotation_* kernels.

Run on a B200 after ``python oracle/build_ref.py`` (which compiles
kernel-source/legacy-v2/src/block_rotation.cu into oracle/_ref/):

    python tests/golden/gen_rotation_golden.py [out.npz]

It launches the reference kernels through oracle/ref_gpu.py on seeded inputs and saves inputs and
outputs to ``tests/golden/rotation_reference.npz`` (or ``out.npz``), which
``tests/test_rotation_cpu.py`` checks the oracle against on the CPU.
"""
import os
import sys

import numpy as np
import torch

sys.path.insert(0, os.path.join(os.path.dirname(__file__), "..", ".."))
from oracle import ref_gpu  # noqa: E402
from oracle import reax_oracle as ro  # noqa: E402

# (M, K, chunk, parts, group, block, threads) - one per reference group shape, small enough to commit
CASES = [(2, 3072, 1024, 3, 1024, 1024, 128), (3, 2304, 2304, 1, 2304, 256, 64), (2, 4096, 1280, 4, 1344, 64, 64),
         (2, 2816, 1408, 2, 1408, 128, 128), (4, 1000, 512, 2, 512, 512, 256), (1, 6144, 3072, 2, 3072, 1024, 64),
         (2, 1536, 512, 3, 512, 64, 64)]


def main(out):
    g = torch.Generator().manual_seed(2024)
    rot = ref_gpu.Rotation()
    arrays = {"cases": np.array(len(CASES))}
    for i, (M, K, chunk, parts, group, block, threads) in enumerate(CASES):
        x = ro.f32_to_bf16(torch.randn(M, K, generator=g).numpy().astype(np.float32))
        centers = (torch.randn(K, generator=g) * 0.05).numpy().astype(np.float32)
        xd = torch.from_numpy(x.view(np.int16)).view(torch.bfloat16).cuda()
        low, scales = rot.prepare(xd, torch.from_numpy(centers).cuda(), chunk, parts, group, block, threads)
        torch.cuda.synchronize()
        arrays.update({f"c{i}_shape": np.array([M, K, chunk, parts, group, block, threads]), f"c{i}_x": x,
                       f"c{i}_centers": centers, f"c{i}_low": low.cpu().numpy(), f"c{i}_scales": scales.cpu().numpy()})
    np.savez_compressed(out, **arrays)
    print("wrote", out)


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.path.join(os.path.dirname(__file__), "rotation_reference.npz"))
