"""GPU parity of the rotated INT8 down projection (reaxv2/rotation.py) against the CPU oracle and the
reference's own rotation_* kernels, compiled from source for sm_100a (oracle/_ref/block_rotation.cubin).

The rotated quantizer's codes and scales are bit-identical: the butterflies add and subtract float32
values in the reference's stage order (index bit 0 first), the scale is a float32 multiply by
fl(1/127) and the codes an IEEE division rounded to nearest even.  The projection (rotated quantizer,
grouped INT8 partials, ordered fold) is then bit-identical as well.
"""
from types import SimpleNamespace

import numpy as np
import pytest
import torch

from oracle import ref_gpu
from oracle import reax_oracle as ro
from tests import helpers as H

pytestmark = pytest.mark.gpu

# (M, K, chunk, parts, group, block): the down projection's input width K = 9216 in three group
# shapes, the GDN output projection's K = 4096 with a group padded past its chunk and past K, a
# 1408-column group, a K that ends inside the last part, a block narrower than a warp, a chunk that is
# no multiple of eight (scalar loads and stores), blocks that span two and four warps, and a group of no
# multiple of 64 columns (the shared-memory kernel).  The second list has launches of many rows, among
# them groups of an odd multiple of 64 columns (the persistent row-walking kernel, with three runs per
# thread and with one), with row counts that leave some CTAs a row fewer than others.
CASES = [(1, 9216, 3072, 3, 3072, 1024), (7, 9216, 2304, 4, 2304, 256), (64, 9216, 1024, 9, 1024, 64),
         (5, 4096, 1280, 4, 1344, 64), (3, 4096, 1408, 3, 1408, 128), (16, 1000, 512, 2, 512, 512),
         (33, 2560, 512, 5, 512, 8), (4, 3000, 700, 5, 768, 256), (9, 5120, 2560, 2, 2560, 512),
         (6, 4096, 2048, 2, 2048, 1024), (2, 500, 96, 6, 96, 32)]
MANY_ROWS = [(1024, 9216, 2304, 4, 2304, 256), (250, 9216, 3072, 3, 3072, 1024), (301, 4096, 1408, 3, 1408, 128),
             (601, 4096, 1280, 4, 1344, 64), (600, 1000, 512, 2, 512, 512), (150, 5000, 1020, 5, 1024, 256),
             (201, 2560, 512, 5, 512, 8), (150, 8192, 2048, 4, 2048, 1024), (300, 9216, 1024, 9, 1024, 64),
             (1501, 1280, 320, 4, 320, 64), (1499, 1216, 304, 4, 320, 32)]


def inputs(M, K, seed):
    g = H.gen(seed)
    x = H.activations(g, M, K)
    centers = (torch.randn(K, generator=g) * 0.05).float()
    return x, centers


@pytest.mark.parametrize("M,K,chunk,parts,group,block", CASES + MANY_ROWS)
def test_rotated_quantizer_vs_oracle(M, K, chunk, parts, group, block):
    from reax_engine_runtime_v3_b200.reaxv2.rotation import quantize_rotated
    x, centers = inputs(M, K, M + K + group + block)
    low, scales = quantize_rotated(x.cuda(), centers.cuda(), chunk, parts, group, block)
    torch.cuda.synchronize()
    lo, sc = ro.prepare_rotated(H.bits(x), centers.numpy(), chunk, parts, group, block)
    assert np.array_equal(scales.cpu().numpy().view(np.int32), sc.view(np.int32))
    assert np.array_equal(low.cpu().numpy(), lo)


def _offset_copy(t, elements):
    """A contiguous copy of t whose data starts `elements` elements past an allocation boundary."""
    buf = torch.empty(t.numel() + elements, dtype=t.dtype, device=t.device)
    view = buf[elements:].view(t.shape)
    view.copy_(t)
    return view


@pytest.mark.parametrize("M,K,chunk,parts,group,block", [(3, 9216, 2304, 4, 2304, 256), (5, 4096, 1408, 3, 1408, 128),
                                                         (4, 4096, 1280, 4, 1344, 64), (600, 9216, 2304, 4, 2304, 256),
                                                         (301, 4096, 1408, 3, 1408, 128),
                                                         (222, 4096, 1280, 4, 1344, 64)])
@pytest.mark.parametrize("x_off,c_off", [(1, 0), (0, 1), (4, 2)])
def test_rotated_quantizer_unaligned_inputs(M, K, chunk, parts, group, block, x_off, c_off):
    """Input rows or centers that do not start on a vector boundary take the scalar loads."""
    from reax_engine_runtime_v3_b200.reaxv2.rotation import quantize_rotated
    x, centers = inputs(M, K, 3 * M + K + x_off + 5 * c_off)
    low, scales = quantize_rotated(_offset_copy(x.cuda(), x_off), _offset_copy(centers.cuda(), c_off), chunk, parts,
                                   group, block)
    torch.cuda.synchronize()
    lo, sc = ro.prepare_rotated(H.bits(x), centers.numpy(), chunk, parts, group, block)
    assert np.array_equal(scales.cpu().numpy().view(np.int32), sc.view(np.int32))
    assert np.array_equal(low.cpu().numpy(), lo)


def _near_half_rows(rows, K, seed):
    """bf16 rows whose rotated values (block 2, zero centers, every odd column zero, so both outputs
    of a pair are +-x) have quotients v / scale within 2^-13 of a half-integer: the codes the kernel
    must take from the division itself rather than from v * (1 / scale)."""
    rng = np.random.default_rng(seed)
    out = np.zeros((rows, K), dtype=np.uint16)
    found = 0
    for r in range(rows):
        top = np.uint16(0x3F80 + rng.integers(0, 0x400))            # the row maximum, in [1, 256)
        top_f = ro.bf16_to_f32(np.array([top], np.uint16))[0]
        scale = np.float32(np.float32(max(top_f, np.float32(1e-12))) * np.float32(np.float32(1) / np.float32(127)))
        cand = np.arange(0x3C00, top, dtype=np.uint16)              # positive bf16 values below the maximum
        q = (ro.bf16_to_f32(cand) / scale).astype(np.float32)
        near = cand[np.abs(np.abs(q - np.floor(q)) - np.float32(0.5)) < np.float32(2.0 ** -13)]
        pick = rng.choice(near, size=min(len(near), K // 2 - 1), replace=False) if len(near) else near
        found += len(pick)
        row = np.zeros(K, dtype=np.uint16)
        row[0] = top
        row[2:2 + 2 * len(pick):2] = pick
        out[r] = row
    return out, found


@pytest.mark.parametrize("M", [256, 700])
def test_rotated_quantizer_near_half_quotients(M):
    from reax_engine_runtime_v3_b200.reaxv2.rotation import quantize_rotated
    K = 512
    xb, found = _near_half_rows(M, K, 11)
    assert found >= 100
    x = H.from_bits(xb)
    centers = torch.zeros(K)
    low, scales = quantize_rotated(x.cuda(), centers.cuda(), K, 1, K, 2)
    torch.cuda.synchronize()
    lo, sc = ro.prepare_rotated(xb, centers.numpy(), K, 1, K, 2)
    # the inputs bite: rounding v * (1 / scale) instead of v / scale changes some of the codes
    v = np.abs(ro.bf16_to_f32(xb))
    naive = np.rint((v * (np.float32(1) / sc[0])[:, None]).astype(np.float32)).astype(np.int64)
    assert (naive != np.abs(lo.astype(np.int64))).any()
    assert np.array_equal(scales.cpu().numpy().view(np.int32), sc.view(np.int32))
    assert np.array_equal(low.cpu().numpy(), lo)


@pytest.mark.skipif(not ref_gpu.available("block_rotation.cubin"), reason="reference rotation kernel not built")
@pytest.mark.parametrize("M,K,chunk,parts,group,block,threads", [
    (1, 9216, 3072, 3, 3072, 1024, 256), (7, 9216, 2304, 4, 2304, 256, 64), (64, 9216, 1024, 9, 1024, 64, 64),
    (5, 4096, 1280, 4, 1344, 64, 64), (3, 4096, 1408, 3, 1408, 128, 128), (16, 1000, 512, 2, 512, 512, 128)])
def test_rotated_quantizer_bit_identical_to_reference_kernel(M, K, chunk, parts, group, block, threads):
    from reax_engine_runtime_v3_b200.reaxv2.rotation import quantize_rotated
    x, centers = inputs(M, K, 7 * M + K + group)
    xd, cd = x.cuda(), centers.cuda()
    low, scales = quantize_rotated(xd, cd, chunk, parts, group, block)
    ref_low, ref_scales = ref_gpu.Rotation().prepare(xd, cd, chunk, parts, group, block, threads)
    torch.cuda.synchronize()
    assert torch.equal(scales.view(torch.int32), ref_scales.view(torch.int32))
    assert torch.equal(low, ref_low)


def rotated_bank(g, K, parts, group, block, N):
    return SimpleNamespace(
        width=K, parts=parts, group=group, block=block, chunk=-(-K // parts), hp=0,
        centers=(torch.randn(K, generator=g) * 0.05).float(),
        low_weight=torch.randint(-127, 128, (N, parts * group), generator=g, dtype=torch.int32).to(torch.int8),
        high_weight=torch.zeros(N, 0, dtype=torch.bfloat16),
        scales=(1e-3 + 9e-3 * torch.rand(parts, N, generator=g)).float(),
        bias=(torch.randn(parts, N, generator=g) * 0.05).float())


@pytest.mark.parametrize("M,K,parts,group,block,N", [(1, 9216, 3, 3072, 1024, 2560), (64, 9216, 4, 2304, 256, 2560),
                                                     (17, 4096, 4, 1024, 64, 2560), (8, 4096, 3, 1408, 128, 512)])
def test_rotated_projection(M, K, parts, group, block, N):
    """The down projection as the runtime calls it (assets.py:82 -> rotation.Native.project), against
    the oracle's composition and against the reference's kernels composed the same way."""
    from reax_engine_runtime_v3_b200.reaxv2.rotation import Native as Rotation
    from reax_engine_runtime_v3_b200.reaxv2.sliced import Native as Sliced
    g = H.gen(M + K + group + N)
    x = H.activations(g, M, K)
    bank = rotated_bank(g, K, parts, group, block, N)
    bd = H.bank_to(bank, "cuda")
    native = Rotation(Sliced(None), None, 128)
    ours = native.project(x.cuda(), bd, "slice_m128n256")
    torch.cuda.synchronize()
    want = ro.rotated_project(H.bits(x), H.bank_numpy(bank))
    assert np.array_equal(H.bits(ours), want)
    if ref_gpu.available("block_rotation.cubin") and ref_gpu.available("sliced_linear8.cubin"):
        threads = 64   # a thread count every reference rotation_* group shape has
        low, scales = ref_gpu.Rotation().prepare(x.cuda(), bd.centers, bank.chunk, parts, group, block, threads)
        empty_a = torch.zeros(M, 0, dtype=torch.bfloat16, device="cuda")
        partials = ref_gpu.Sliced8().partials(low, bd.low_weight, empty_a, bd.high_weight, scales, bd.scales,
                                              bd.bias, group, 0, parts)
        torch.cuda.synchronize()
        assert np.array_equal(H.bits(ours), ro.reduce_partials(H.bits(partials)))


def test_asset_policy_runs_the_rotated_projection(tmp_path):
    """A frozen bank loaded by the asset drop-in (reaxv2/assets.py) and routed by its policy runs the rotated
    projection on the GPU with the oracle's bits."""
    from tests.test_assets_cpu import core_with_layers, write_assets
    from reax_engine_runtime_v3_b200.reaxv2.assets import Assets
    g = H.gen(4242)
    K, parts, group, block, N, M = 2048, 2, 1024, 64, 512, 17
    bank = rotated_bank(g, K, parts, group, block, N)
    payload = {"schema": 1, "checkpoint_start": 12, "gate_up": {}, "projections": {(14, "down", K): vars(bank)},
               "chunk_for": {(14, "down", 64): K}, "projection_routes": {},
               "rotation_routes": {("down", 64, 16, 8): dict(kernel="slice_m128n256", drop=0, threads=128)},
               "rotation_cap": 8}
    write_assets(tmp_path, payload)
    assets = Assets(tmp_path)
    assets.bind(core_with_layers(32))
    x = H.activations(g, M, K)
    out = assets.policy.project(14, "down", x.cuda(), 64)
    torch.cuda.synchronize()
    assert np.array_equal(H.bits(out), ro.rotated_project(H.bits(x), H.bank_numpy(bank)))
