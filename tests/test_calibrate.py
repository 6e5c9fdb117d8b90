"""`unikern calibrate` on the host (uk_calibrate): the ledger's measured rows
under an HCS fingerprint -> the effective host link bandwidth -> a calibrated
HCS.  The cases and numbers are the reference's own (tests/acceptance.cpp:
778-870 for the median and the export round trip, :916-1000 for the
unified-memory gate)."""
import json
import re

import pytest

import unikern_b200.abi as abi

B200 = (abi.SAMPLES / "hcs_nvidia_b200.json").read_text()


def fingerprint(hcs_json):
    return abi.kml_describe('{"op":"gemm","dtype":"fp32","dims":[8,8,8]}', hcs_json)["hcs_fingerprint"]


def unified_hcs(link=600):
    return json.dumps({"vendor": "apple", "device": "unified test device", "unified_memory": True,
                       "link_bw_gbps": link, "flops_gflops": 20000, "compute_units": 40,
                       "tiers": [{"name": "unified", "bytes": 68719476736, "bw_gbps": 400}]})


def discrete_hcs(link=32):
    return json.dumps({"vendor": "amd", "device": "discrete test device", "unified_memory": False,
                       "link_bw_gbps": link, "flops_gflops": 22000, "compute_units": 36,
                       "tiers": [{"name": "vram", "bytes": 8589934592, "bw_gbps": 512}]})


def test_median_of_usable_rows(tmp_path):
    # gemm fp32 1024^3 -> 3 * 1024^2 * 4 = 12582912 B: copy 1.5 ms -> 8.388608,
    # copy 2.5 ms -> 5.0331648 GB/s; a 6-field row (no kernel time), a row with
    # measured <= kernel, an unmeasured row and another HCS's row are unusable
    fp = fingerprint(B200)
    led = tmp_path / "l.jsonl"
    led.write_text(f"gemm:fp32:1024x1024x1024|{fp}|th1\t0.5\t2.0\t0.5\t128\t128\tp\n"
                   f"gemm:fp32:1024x1024x1024|{fp}|th2\t0.5\t3.0\t0.5\t128\t128\tp\n"
                   f"gemm:fp32:1024x1024x1024|{fp}|th3\t0.5\t2.0\t128\t128\tp\n"
                   f"gemm:fp32:1024x1024x1024|{fp}|th4\t0.5\t0.4\t0.5\t128\t128\tp\n"
                   f"gemm:fp32:512x512x512|{fp}|th5\t0.5\t0\t0.1\t128\t128\tp\n"
                   f"gemm:fp32:1024x1024x1024|fpB|th6\t0.5\t1.1\t0.5\t128\t128\tp\n"
                   f"#VIOLATION\tgemm:fp32:1024x1024x1024|{fp}|th1\t0.5\t0.01\t1\t4\t0\n")
    rc, cal, out = abi.calibrate(B200, str(led))
    assert rc == 0, out
    assert "usable_rows=2" in out
    bw = json.loads(cal)["link_bw_gbps"]
    assert 6.7108 < bw < 6.7109
    assert "CALIBRATED link_bw_gbps 55 -> 6.71089 constants_version 1 -> 2" in out
    # a slower link than declared: the predicted time of the demo tree grows
    before, after = map(float, re.search(r"PREDICTED demo c_ms (\S+) -> (\S+)", out).groups())
    assert after > before


def test_calibrated_hcs_round_trips(tmp_path):
    fp = fingerprint(B200)
    led = tmp_path / "l.jsonl"
    led.write_text(f"gemm:fp32:512x512x512|{fp}|thA\t0.5\t1.0\t0.5\t128\t128\tp\n")
    rc, cal, out = abi.calibrate(B200, str(led))
    assert rc == 0
    h = json.loads(cal)
    assert h["constants_version"] == 2 and h["toolchain"] == "cuda-12.9"
    assert [t["confidence"] for t in h["tiers"]] == ["official", "predicted"]
    assert 6.2914 < h["link_bw_gbps"] < 6.2915   # 3145728 B / 0.5 ms
    # the export imports again and keeps every modelled field but the link
    src = json.loads(B200)
    for k in ("vendor", "device", "unified_memory", "flops_gflops", "compute_units"):
        assert h[k] == src[k]
    assert fingerprint(cal) != fingerprint(B200)
    # calibrating the export again bumps the version once more
    led2 = tmp_path / "l2.jsonl"
    led2.write_text(f"gemm:fp32:512x512x512|{fingerprint(cal)}|thA\t0.5\t1.0\t0.5\t128\t128\tp\n")
    rc, cal2, _ = abi.calibrate(cal, str(led2))
    assert rc == 0 and json.loads(cal2)["constants_version"] == 3


def test_constants_version_is_provenance_only():
    j1 = json.loads(discrete_hcs())
    j3 = dict(j1, constants_version=3)
    assert fingerprint(json.dumps(j1)) == fingerprint(json.dumps(j3))


def test_unified_memory_gate(tmp_path):
    uni = unified_hcs(600)
    row = f"gemm:fp32:512x512x512|{fingerprint(uni)}|thA\t0.5\t1.0\t0.5\t128\t128\tp\n"
    led = tmp_path / "uni.jsonl"
    led.write_text(row)
    empty = tmp_path / "empty.jsonl"
    # arm 1: refused by the gate before the ledger is read
    rc, cal, out = abi.calibrate(uni, str(empty))
    assert rc == 3 and "CALIBRATE SKIP: scenario A" in out and cal == ""
    # arm 2: with the flag the empty ledger is what stops it
    rc, _, out = abi.calibrate(uni, str(empty), allow_unified=True)
    assert rc == 3 and "CALIBRATE SKIP: scenario A" not in out and "no measured rows" in out
    # arm 3: with the flag and a measured row it calibrates and keeps the scenario
    rc, cal, out = abi.calibrate(uni, str(led), allow_unified=True)
    assert rc == 0 and "CALIBRATED link_bw_gbps 600 -> 6.29146" in out
    h = json.loads(cal)
    assert 6.2914 < h["link_bw_gbps"] < 6.2915 and h["constants_version"] == 2 and h["unified_memory"] is True
    # arm 4: a discrete HCS is not gated
    dis = discrete_hcs(32)
    led_d = tmp_path / "dis.jsonl"
    led_d.write_text(f"gemm:fp32:512x512x512|{fingerprint(dis)}|thA\t0.5\t1.0\t0.5\t128\t128\tp\n")
    rc, cal, out = abi.calibrate(dis, str(led_d))
    assert rc == 0 and "CALIBRATE SKIP" not in out and "CALIBRATED link_bw_gbps 32 -> 6.29146" in out


def test_no_usable_rows_and_bad_hcs(tmp_path):
    fp = fingerprint(B200)
    led = tmp_path / "l.jsonl"
    led.write_text(f"gemm:fp32:512x512x512|{fp}|thA\t0.5\t1.0\t128\t128\tp\n")  # no kernel time
    rc, _, out = abi.calibrate(B200, str(led))
    assert rc == 3 and "no usable rows" in out
    rc, _, out = abi.calibrate('{"vendor":"nvidia"}', str(led))
    assert rc == 2 and "HCS rejected" in out
