"""The Blackwell GEMM solver (uk_cuda_solve_plan; uk::solve_gemm in
csrc/uk_plan.cuh), CPU only: the re-target of the reference's sketch ->
feasible -> cost -> lexicographic argmin (src/solver.cpp:14-186) to this
library's kernel families.  The argmin must change with the shape for the
reasons the cost model encodes, be deterministic, agree with the tile plan the
ledger records, and reach the solve transcript."""
import pytest

import unikern_b200.abi as abi

B200_HCS = (abi.SAMPLES / "hcs_nvidia_b200.json").read_text()


@pytest.mark.parametrize("M,N,K,f16,family,tile,ks", [
    (8192, 8192, 8192, True, "tcgen05-2sm", (256, 256), 1),   # the headline: SM pairs
    (128, 4096, 4096, True, "tcgen05-1sm", (128, 256), 1),    # one 128-row block: the pair is infeasible
    # 640 rows: 3 pair rows (768, 17% idle) against 5 single rows; with 59
    # column tiles the single-SM grid fits 2 waves on 148 SMs where the
    # pair grid needs 3 on 74 pairs
    (640, 15104, 4096, True, "tcgen05-1sm", (128, 256), 1),
    (640, 16384, 4096, True, "tcgen05-2sm", (256, 256), 1),   # 64 column tiles: 3 waves either way
    # 512^3: 64 tiles of 64 x 64, 8 x 8 per thread, K split over 4-CTA clusters
    # (16.7 us against 18.4 for 32 x 64 tiles split 4 ways, L2 flushed)
    (512, 512, 512, False, "ffma", (64, 64), 4),
    (256, 256, 256, False, "ffma", (32, 64), 4),
    (2048, 2048, 2048, False, "tcgen05-2sm-3xtf32", (256, 256), 1),
    (4096, 4096, 4096, False, "tcgen05-2sm-3xtf32", (256, 256), 1),
    (4096, 4096, 4090, False, "ffma", (128, 128), 1),         # K % 32: no split-tf32 candidate
    # mid sizes: the 64 x 64 tile with 8 x 8 per thread and K split over 4
    # CTAs (measured 114 against 147 us for the 32 x 64 split, L2 flushed)
    (1000, 3000, 700, False, "ffma", (64, 64), 4),
])
def test_argmin_changes_with_shape(M, N, K, f16, family, tile, ks):
    p = abi.solve_plan(M, N, K, f16, sms=148)
    assert (p["family"], p["tile"], p["k_split"]) == (family, tile, ks), p
    # the tile plan the ledger records is the argmin's tile
    assert abi.tile_plan("gemm", (M, N, K), f16, sms=148)[:2] == tile


def test_without_the_tensor_cores_fp32_stays_on_ffma():
    p = abi.solve_plan(4096, 4096, 4096, False, sms=148, allow_tc=False)
    assert p["family"] == "ffma" and p["tile"] == (128, 128) and p["feasible"] == 8
    assert abi.solve_plan(4096, 4096, 4096, False, sms=148)["feasible"] == 9
    # without them, 2048^3 takes the 8 x 8 split tiles (measured 399 against
    # 462 us for 128 x 128, whose 256 tiles are 1.7 waves on 148 SMs)
    p = abi.solve_plan(2048, 2048, 2048, False, sms=148, allow_tc=False)
    assert p["tile"] == (64, 64) and p["k_split"] == 4


def test_smaller_parts_shift_the_choice():
    # 256^3 on 148 SMs: the 64 CTAs of the 8 x 8 split leave most SMs idle
    # and the 32 x 64 tiles split 4 ways win; on a 16-SM part every SM is
    # busy either way and the 8 x 8 micro-tiles' higher FFMA rate wins
    p = abi.solve_plan(256, 256, 256, False, sms=148)
    assert p["tile"] == (32, 64) and p["k_split"] == 4
    p = abi.solve_plan(256, 256, 256, False, sms=16)
    assert p["tile"] == (64, 64) and p["k_split"] == 4


def test_deterministic_and_costed():
    a = abi.solve_plan(1000, 3000, 700, False, sms=148)
    assert all(abi.solve_plan(1000, 3000, 700, False, sms=148) == a for _ in range(5))
    # predicted time grows with the work
    t = [abi.solve_plan(n, n, n, True, sms=148)["ns"] for n in (1024, 2048, 4096, 8192)]
    assert t == sorted(t) and t[-1] > 6 * t[-2]


def test_solve_transcript_carries_the_grid():
    rc, out = abi.solve_kml(B200_HCS, '{"op":"gemm","dtype":"fp16","dims":[640,15104,4096]}', None)
    assert rc == 0 and "tile=128x256" in out and "|X|=2" in out and "kernel=tcgen05-1sm" in out, out
    rc, out = abi.solve_kml(B200_HCS, '{"op":"gemm","dtype":"fp32","dims":[512,512,512]}', None)
    assert rc == 0 and "|X|=8" in out and "kernel=ffma k_split=4" in out, out
