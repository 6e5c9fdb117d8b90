"""Workspace and ring size queries and argument checks of the C ABI that need
no GPU (the library reports a 148-SM B200 when no device is visible, the
count it then plans for)."""
import unikern_b200.abi as abi

KIB = 1024
PARTIAL_TILE = 2 * 256 * 128 * 4   # one split item's fp32 partials (2 CTAs x 256 channels x 128 pixels)


def align(n):
    return -(-n // 256) * 256


def test_conv_workspace_holds_pairs_and_last_round_partials():
    L = abi.lib()
    N, H, W, C, Oc = 32, 56, 56, 256, 256
    base = 2 * align(N * H * W * C * 4) + 2 * align(Oc * 9 * C * 4)
    # 448 pair tiles on 74 pairs: 4 in the last round, each split 18 ways
    assert L.uk_cuda_conv2d_workspace_size(N, H, W, C, 3, 3, Oc, 1, abi.UK_CONV_NCHW) == base + 4 * 18 * PARTIAL_TILE
    # C not a multiple of 32: the FFMA kernel, no workspace
    assert L.uk_cuda_conv2d_workspace_size(N, H, W, 8, 3, 3, Oc, 1, abi.UK_CONV_NCHW) == 0


def test_fp16_conv_workspace():
    L = abi.lib()
    # KML layout: read in place; the workspace is only the optional partials
    # (14 tiles, all in the last round, 5 ways each: 36 k-steps / 4 caps at 9)
    assert L.uk_cuda_conv2d_f16_workspace_size(1, 58, 58, 256, 3, 3, 256, 0, abi.UK_CONV_KML) == 14 * 5 * PARTIAL_TILE
    assert L.uk_cuda_conv2d_f16_workspace_size(1, 58, 58, 96, 3, 3, 256, 0, abi.UK_CONV_KML) == 0   # C % 64


def test_gemm_f32_tensor_core_workspace():
    L = abi.lib()
    pairs = 2 * 2 * align(4096 * 4096 * 4)
    # 256 tiles: 34 in the last round, each split in two
    assert L.uk_cuda_gemm_f32_workspace_size(4096, 4096, 4096) == pairs + 34 * 2 * PARTIAL_TILE
    # 1024 tiles: 62 in the last round, no room to split
    assert L.uk_cuda_gemm_f32_workspace_size(8192, 8192, 8192) == 2 * 2 * align(8192 * 8192 * 4)
    assert L.uk_cuda_gemm_f32_prefers_tc(4096, 4096, 4096) == 1
    assert L.uk_cuda_gemm_f32_prefers_tc(4096, 4096, 4090) == 0


def test_streamed_ring_sizes():
    L = abi.lib()
    M, N, K, rows = 4096, 1024, 1024, 1024
    ffma = L.uk_cuda_gemm_streamed_ring_size(M, N, K, 2, rows)
    tc = L.uk_cuda_gemm_streamed_ring_size(M, N, K, 0, rows)
    f16 = L.uk_cuda_gemm_streamed_ring_size(M, N, K, 1, rows)
    assert ffma >= 2 * rows * (K + N) * 4
    assert tc == ffma + 2 * align(N * K * 4) + 2 * align(rows * K * 4)   # + tf32 pairs of B^T and one A block
    assert f16 >= 2 * rows * (K + N) * 2 and f16 < ffma
    assert L.uk_cuda_gemm_streamed_ring_size(M, N, K, 3, rows) == 0


def test_argument_checks_before_any_device_work():
    L = abi.lib()
    assert L.uk_cuda_gemm_streamed(None, None, None, None, None, 0, 8, 8, 8, 5, 8, None) == 2
    assert L.uk_cuda_gemm_streamed(None, None, None, None, None, 0, 8, 8, 8, 1, 0, None) == 2
    assert L.uk_cuda_selftest_wait(0, 10, None, None) == 2
    assert L.uk_cuda_selftest_wait(0, 2_000_000_000, None, None) == 2
    assert L.uk_cuda_reduce_f32_width(None, None, 1, 8, 0, None, 0, None) == 2
    assert L.uk_cuda_reduce_f16_width(None, None, 1, 8, 0, None, 0, None) == 2
    assert b"width" in L.uk_cuda_last_error()
