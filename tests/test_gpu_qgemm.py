"""GPU test of the int8 tensor-core product behind the W8 projections (tcgen05.mma kind::i8): the int32
accumulators of codes x activation digits must equal an exact integer product computed with numpy, and
the per-token steps must equal the fp32 formula bit for bit. The fp32 results of the full projections are
covered by the layer tests against the oracle (test_gpu_dropin.py, test_gpu_engine.py)."""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

DIGIT_RANGE = np.float32(8355710.0)


def digits_numpy(x: np.ndarray):
    """x [nt][k] fp32 -> (step [nt] fp32, digits [3][nt][k] int64), the same fp32 operations as the kernel."""
    x = x.astype(np.float32)
    mx = np.abs(x).max(axis=1)
    step = np.where(mx > 0, mx / DIGIT_RANGE, np.float32(1.0)).astype(np.float32)
    X = np.rint(x / step[:, None]).astype(np.int64)
    d0 = ((X + 128) & 255) - 128
    r1 = (X - d0) >> 8
    d1 = ((r1 + 128) & 255) - 128
    d2 = (r1 - d1) >> 8
    assert np.all(d0 + 256 * d1 + 65536 * d2 == X)
    assert max(abs(d).max() for d in (d0, d1, d2)) <= 128
    return step, np.stack([d0, d1, d2])


def run_case(rows, k, nt, seed, special=None):
    import torch

    from work_llm_accelerator_b200 import host

    rng = np.random.default_rng(seed)
    codes = rng.integers(-127, 128, size=(rows, k), dtype=np.int8)
    codes[0, :] = 127                       # extreme rows: the largest accumulator magnitudes
    codes[rows - 1, :] = -127
    codes[1, ::7] = -128
    x = rng.standard_normal((nt, k)).astype(np.float32)
    x[:, rng.integers(0, k, 3)] *= 50.0     # outliers set the step
    if special == "zero_row":
        x[nt - 1, :] = 0.0
    if special == "one_hot":
        x[0, :] = 0.0
        x[0, k // 2] = -3.25
    if special == "same_sign":
        x = np.abs(x)
    step_ref, d = digits_numpy(x)
    acc_ref = np.zeros((rows, 12), np.int64)
    c64 = codes.astype(np.int64)
    for di in range(3):
        acc_ref[:, 4 * di:4 * di + nt] = c64 @ d[di].T
    assert np.abs(acc_ref).max() < 2**31

    dev = torch.device("cuda")
    codes_d = torch.from_numpy(codes).to(dev)
    x_d = torch.from_numpy(x).to(dev)
    acc_d = torch.full((rows, 12), -7, dtype=torch.int32, device=dev)
    step_d = torch.zeros(nt, dtype=torch.float32, device=dev)
    host.w8_digit_products(codes_d.data_ptr(), rows, k, x_d.data_ptr(), nt, acc_d.data_ptr(), step_d.data_ptr(),
                           torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert host.kernel_error(reset=True) == 0
    acc = acc_d.cpu().numpy().astype(np.int64)
    np.testing.assert_array_equal(step_d.cpu().numpy().view(np.uint32), step_ref.view(np.uint32))
    bad = np.argwhere(acc != acc_ref)
    assert bad.size == 0, f"{len(bad)} mismatches, first {bad[:4].tolist()}"


@pytest.mark.parametrize("rows,k,nt,special", [
    (128, 128, 1, None),          # one tile, one K block
    (256, 1536, 4, None),         # o_proj / q|k|v shape: split-K over 4 CTAs per tile
    (2048, 1536, 3, "zero_row"),  # q|k|v rows; a token whose activations are all zero
    (1536, 8960, 1, None),        # down_proj shape: 70 K blocks in one CTA per tile
    (1536, 8960, 2, "one_hot"),
    (4096, 1536, 2, "same_sign"), # more rows than the split-K scratch: one CTA per tile
])
def test_digit_products_exact(built_libs, gpu_available, rows, k, nt, special):
    if not gpu_available:
        pytest.fail("no CUDA device")
    run_case(rows, k, nt, seed=rows + k + nt, special=special)


def test_digit_products_repeat_leaves_scratch_clean(built_libs, gpu_available):
    """The split-K scratch is zero again after every call: the same call twice gives the same result."""
    if not gpu_available:
        pytest.fail("no CUDA device")
    for _ in range(3):
        run_case(512, 1536, 4, seed=5)


def test_digit_products_rejects_bad_shapes(built_libs, gpu_available):
    import torch

    from work_llm_accelerator_b200 import host

    if not gpu_available:
        pytest.fail("no CUDA device")
    a = torch.zeros(4096, dtype=torch.int32, device="cuda")
    for rows, k, nt in [(100, 128, 1), (128, 100, 1), (128, 128, 5), (128, 128, 0)]:
        with pytest.raises(host.EngineError):
            host.w8_digit_products(a.data_ptr(), rows, k, a.data_ptr(), nt, a.data_ptr(), a.data_ptr())


@pytest.mark.parametrize("rows,k,nt", [
    (128, 128, 1),      # one tile, one K block, one token
    (256, 1536, 130),   # two token tiles, the second ragged
    (2048, 1536, 300),  # q|k|v rows, three token tiles
    (2048, 1536, 64),   # one 64-token tile, few row tiles: K split over 8-CTA clusters
    (9728, 1536, 33),   # one 64-token tile, many row tiles: the CTA-pair form, one wave (two MMA issuers)
    (9728, 1536, 200),  # four token tiles: CTA pairs beyond one wave (one issuer, two CTAs per SM)
    (128, 8960, 129),   # down_proj K, ragged tokens
    (256, 8960, 2433),  # many token tiles: the CTA-pair form (256-row tiles), ragged tokens
])
def test_digit_planes_exact(built_libs, gpu_available, rows, k, nt):
    """Many-token tensor-core path (prefill / batched projections): three int32 planes per output, exact."""
    import torch

    from work_llm_accelerator_b200 import host

    if not gpu_available:
        pytest.fail("no CUDA device")
    rng = np.random.default_rng(rows * 7 + nt)
    codes = rng.integers(-127, 128, size=(rows, k), dtype=np.int8)
    codes[0, :] = 127
    codes[rows - 1, :] = -128
    x = rng.standard_normal((nt, k)).astype(np.float32)
    x[:, rng.integers(0, k, 5)] *= 40.0
    x[nt // 2, :] = 0.0  # an all-zero token row (step 1)
    step_ref, d = digits_numpy(x)
    dev = torch.device("cuda")
    if rows * k * nt <= 2**31:
        c64 = codes.astype(np.int64)
        acc_ref = np.stack([d[p] @ c64.T for p in range(3)])  # [3][nt][rows]
    else:  # float64 products and sums of these integers are exact (|sum| < 2^31 << 2^53)
        c_f = torch.from_numpy(codes.astype(np.float64)).to(dev)
        acc_ref = np.stack([(torch.from_numpy(d[p].astype(np.float64)).to(dev) @ c_f.T).cpu().numpy()
                            for p in range(3)]).astype(np.int64)
    assert np.abs(acc_ref).max() < 2**31
    codes_d = torch.from_numpy(codes).to(dev)
    x_d = torch.from_numpy(x).to(dev)
    acc_d = torch.full((3, nt, rows), -7, dtype=torch.int32, device=dev)
    step_d = torch.zeros(nt, dtype=torch.float32, device=dev)
    host.w8_digit_planes(codes_d.data_ptr(), rows, k, x_d.data_ptr(), nt, acc_d.data_ptr(), step_d.data_ptr(),
                         torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert host.kernel_error(reset=True) == 0
    np.testing.assert_array_equal(step_d.cpu().numpy().view(np.uint32), step_ref.view(np.uint32))
    acc = acc_d.cpu().numpy().astype(np.int64)
    bad = np.argwhere(acc != acc_ref)
    assert bad.size == 0, f"{len(bad)} mismatches, first {bad[:4].tolist()}"
