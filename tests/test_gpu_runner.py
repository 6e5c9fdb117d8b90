"""The nvidia:cuda runner on the GPU: `uk_run_kml` runs a KML declaration the
way the reference's `unikern run` runs one on its own backends (verify
instance, timing, UNIKERN_RESULT line, ledger commit; src/main.cpp:346-570,
src/runner_ocl.cpp).

The verify instances are the reference's own (sawtooth operands that keep
every fp32 partial sum exact, src/codegen_hip.cpp:604-605, :2167, :2338):
gemm/conv/reduce/channelscale must come back with max_rel = 0, as the
reference's published runs do; softmax and rmsnorm within a few ulps.
"""
import pytest

import unikern_b200.abi as abi

pytestmark = pytest.mark.gpu
HCS = (abi.SAMPLES / "hcs_nvidia_b200.json").read_text()


@pytest.fixture(scope="module", autouse=True)
def cuda():
    import torch
    assert torch.cuda.is_available()
    torch.cuda.set_device(0)


CASES = [
    ('{"op":"gemm","dtype":"fp32","dims":[512,512,512],"tile_m":64,"tile_n":128,"layout":"NT"}', 0.0),
    ('{"op":"gemm","dtype":"fp16","dims":[512,512,512]}', 2 ** -11),   # one f16 rounding of an exact sum
    ('{"op":"conv","dtype":"fp32","dims":[58,58,256,3,3,256]}', 0.0),
    ('{"op":"reduce","dtype":"fp32","dims":[1048576]}', 0.0),
    ('{"op":"softmax","dtype":"fp32","dims":[65536,256]}', 1e-6),
    ('{"op":"rmsnorm","dtype":"fp32","dims":[4096,1000]}', 1e-6),
    ('{"op":"channelscale","dtype":"fp32","dims":[65536,256]}', 0.0),
    # the fp16 widening (refused by the reference): one f16 rounding of the
    # fp32 result, channelscale exact on the sawtooth operands
    ('{"op":"softmax","dtype":"fp16","dims":[65536,256]}', 2 ** -10),
    ('{"op":"rmsnorm","dtype":"fp16","dims":[4096,1000]}', 2 ** -10),
    ('{"op":"channelscale","dtype":"fp16","dims":[65536,256]}', 0.0),
    ('{"op":"conv","dtype":"fp16","dims":[58,58,256,3,3,256]}', 2 ** -10),
    ('{"op":"reduce","dtype":"fp16","dims":[1048576]}', 0.0),          # 16384 is exact in binary16
]


@pytest.mark.parametrize("kml,max_rel", CASES, ids=lambda v: v[:30] if isinstance(v, str) else "")
def test_run_verifies_and_commits(tmp_path, kml, max_rel):
    ledger = tmp_path / "ledger.jsonl"
    rc, out = abi.run_kml(HCS, kml, str(ledger))
    assert rc == 0, out
    tok = abi.result_tokens(out)
    assert tok["backend"] == "nvidia:cuda" and tok["verify"] == "PASS", out
    assert float(tok["max_rel"]) <= max_rel, out
    assert float(tok["kernel_ms"]) > 0 and float(tok["measured_ms"]) >= float(tok["kernel_ms"])
    assert tok["mode"] == "resident" and tok["migrations"] == "0" and int(tok["checks"]) >= 4
    assert int(tok["vram_total"]) > 100 * 2 ** 30
    d = abi.kml_describe(kml, HCS)
    rows = [r.split("\t") for r in ledger.read_text().splitlines()]
    assert len(rows) == 1 and rows[0][0] == d["ledger_key"]
    assert float(rows[0][2]) == pytest.approx(float(tok["measured_ms"]), rel=1e-5)
    assert "x".join(rows[0][4:6]) == d["tile"]
    assert "LEDGER COMMIT predicted_ms=" in out
    # the second run hits the row and appends its own measurement
    rc, out = abi.run_kml(HCS, kml, str(ledger))
    assert rc == 0 and "LEDGER HIT" in out and len(ledger.read_text().splitlines()) == 2


@pytest.mark.parametrize("kml", [
    '{"op":"gemm","dtype":"fp16","dims":[8192,8192,8192]}',
    '{"op":"reduce","dtype":"fp32","dims":[134217728]}',
    '{"op":"softmax","dtype":"fp32","dims":[8192,16384]}',
    '{"op":"rmsnorm","dtype":"fp32","dims":[8192,16384]}',
], ids=["gemm_f16_8192", "reduce_2^27", "softmax_8192x16384", "rmsnorm_8192x16384"])
def test_baseline_sizes_verify(kml):
    rc, out = abi.run_kml(HCS, kml, None, write_ledger=False)
    assert rc == 0 and "VERIFY PASS (no ledger write)" in out, out
    tok = abi.result_tokens(out)
    assert tok["verify"] == "PASS"
    if "fp16" in kml:
        assert tok["dtype"] == "fp16"


def test_verify_mode_writes_no_ledger(tmp_path):
    ledger = tmp_path / "ledger.jsonl"
    rc, out = abi.run_kml(HCS, '{"op":"reduce","dtype":"fp32","dims":[4096]}', str(ledger), write_ledger=False)
    assert rc == 0 and "VERIFY PASS" in out
    assert not ledger.exists()


def test_oversized_payload_is_refused_when_b_does_not_fit(tmp_path):
    # B alone is 262144^2 fp32 = 256 GiB: beyond 0.85 x HBM, so not even the
    # streamed GEMM (B resident) can run it
    import sqlite3
    ledger = tmp_path / "ledger.sqlite3"
    rc, out = abi.run_kml(HCS, '{"op":"gemm","dtype":"fp32","dims":[1024,262144,262144]}', str(ledger))
    assert rc == 1 and "UNIKERN_ERROR what=stream_refused" in out
    with sqlite3.connect(ledger) as db:  # opened (as the reference opens it), nothing committed
        assert db.execute("SELECT count(*) FROM solutions").fetchone()[0] == 0


def small_vram_hcs(mib):
    import json
    h = json.loads(HCS)
    for t in h["tiers"]:
        if t["name"] == "vram":
            t["bytes"] = mib << 20
    return json.dumps(h)


@pytest.mark.parametrize("kml,rows,max_rel", [
    ('{"op":"gemm","dtype":"fp16","dims":[4096,1024,1024]}', 1280, 2 ** -11),
    ('{"op":"gemm","dtype":"fp32","dims":[2048,1024,1024]}', 512, 0.0),
], ids=["fp16_4096x1024x1024", "fp32_2048x1024x1024"])
def test_payload_beyond_the_device_tier_streams(tmp_path, kml, rows, max_rel):
    # a 16 MiB device tier models a device the operands do not fit: the GEMM
    # runs streamed (scenario B), verifies through the ring and commits
    hcs = small_vram_hcs(16)
    d = abi.kml_describe(kml, hcs)
    assert "placement: streamed" in d["placement"] and f"{rows}-row blocks" in d["placement"]
    ledger = tmp_path / "ledger.jsonl"
    rc, out = abi.run_kml(hcs, kml, str(ledger))
    assert rc == 0, out
    tok = abi.result_tokens(out)
    assert tok["verify"] == "PASS" and float(tok["max_rel"]) <= max_rel, out
    assert tok["mode"] == "streamed" and tok["stream_path"] == "pinned", out
    assert float(tok["kernel_ms"]) > 0 and float(tok["measured_ms"]) > 0
    assert float(tok["payload_mb"]) > 0.85 * 16
    rows_ = [r.split("\t") for r in ledger.read_text().splitlines()]
    assert len(rows_) == 1 and rows_[0][0] == d["ledger_key"] and "streamed" in rows_[0][-1]
    assert abi.lib().uk_cuda_pipeline_fault() == 0


def test_streamed_refused_for_non_gemm(tmp_path):
    rc, out = abi.run_kml(small_vram_hcs(16), '{"op":"softmax","dtype":"fp32","dims":[8192,1024]}',
                          str(tmp_path / "l"))
    assert rc == 1 and "UNIKERN_ERROR what=stream_refused" in out


def test_calibrate_from_measured_runs(tmp_path):
    # resident runs record measured (upload + kernel + download) and kernel
    # time; calibration turns their difference into the host link bandwidth
    import json
    ledger = tmp_path / "ledger.jsonl"
    for kml in ('{"op":"gemm","dtype":"fp32","dims":[2048,2048,2048]}',
                '{"op":"gemm","dtype":"fp16","dims":[4096,4096,4096]}',
                '{"op":"gemm","dtype":"fp16","dims":[8192,4096,2048]}'):
        rc, out = abi.run_kml(HCS, kml, str(ledger))
        assert rc == 0, out
    rc, cal, out = abi.calibrate(HCS, str(ledger))
    assert rc == 0, out
    assert "usable_rows=3" in out
    bw = json.loads(cal)["link_bw_gbps"]
    assert 2.0 < bw < 1000.0, out   # a page-locked host link, PCIe or C2C
    assert json.loads(cal)["constants_version"] == 2


def test_reduce_width_knob(tmp_path, monkeypatch):
    # UK_REDUCE_WIDTH pins the pass-1 width and is reported; a value outside
    # [256, n] is refused, never silently dropped (src/codegen_hip.cpp:874-908)
    kml = '{"op":"reduce","dtype":"fp32","dims":[1048576]}'
    rc, out = abi.run_kml(HCS, kml, None, write_ledger=False)
    assert rc == 0 and "UNIKERN_INFO reduce_width source=plan" in out, out
    monkeypatch.setenv("UK_REDUCE_WIDTH", "4096")
    rc, out = abi.run_kml(HCS, kml, None, write_ledger=False)
    assert rc == 0 and "UNIKERN_INFO reduce_width source=env width=4096 cap=0 n=1048576" in out, out
    assert abi.result_tokens(out)["max_rel"] == "0.000000e+00"
    for bad in ("100", "2000000", "abc"):
        monkeypatch.setenv("UK_REDUCE_WIDTH", bad)
        rc, out = abi.run_kml(HCS, kml, str(tmp_path / "l.jsonl"), write_ledger=True)
        assert rc == 1 and "UNIKERN_ERROR what=reduce_width_pin_unfit value=" + bad in out, out
        assert not (tmp_path / "l.jsonl").exists()


def test_stream_path_knob(tmp_path, monkeypatch):
    # UK_GEMM_STREAM_PATH: pinned (the only arm here) is accepted and reported;
    # mmap and unknown values are refused (src/codegen_hip.cpp:1338-1355)
    kml = '{"op":"gemm","dtype":"fp16","dims":[4096,1024,1024]}'
    monkeypatch.setenv("UK_GEMM_STREAM_PATH", "pinned")
    rc, out = abi.run_kml(small_vram_hcs(16), kml, None, write_ledger=False)
    assert rc == 0 and "UNIKERN_INFO mode=streamed shards=4 shard_rows=1280" in out and "source=env" in out, out
    for bad in ("mmap", "zerocopy"):
        monkeypatch.setenv("UK_GEMM_STREAM_PATH", bad)
        rc, out = abi.run_kml(small_vram_hcs(16), kml, None, write_ledger=False)
        assert rc == 1 and "UNIKERN_ERROR what=stream_path_pin_unfit val=" + bad in out, out


def test_run_commits_an_sqlite_row_both_tools_read(tmp_path):
    # the reference's default ledger is SQLite (src/main.cpp:37, :61-70): a
    # verified run's row is a HIT for the reference's own lookup, a second
    # run is a HIT here that replaces the row, and a row the reference
    # commits is a HIT for uk_run_kml
    import ctypes as C
    import sqlite3

    from oracle import oracle as O
    ledger = tmp_path / "ledger.sqlite3"
    kml = '{"op":"gemm","dtype":"fp32","dims":[512,512,512]}'
    rc, out = abi.run_kml(HCS, kml, str(ledger))
    assert rc == 0 and "LEDGER COMMIT" in out, out
    with sqlite3.connect(ledger) as db:
        rows = db.execute("SELECT key, c_ms, measured_ms, kernel_ms, tm, tn FROM solutions").fetchall()
    assert len(rows) == 1 and rows[0][0] == abi.kml_describe(kml, HCS)["ledger_key"]
    assert rows[0][2] > rows[0][3] > 0  # measured_ms (e2e) > kernel_ms > 0
    rc, out = abi.run_kml(HCS, kml, str(ledger))
    assert rc == 0 and "LEDGER HIT" in out, out
    with sqlite3.connect(ledger) as db:
        assert db.execute("SELECT count(*) FROM solutions").fetchone()[0] == 1
    r = O.ref()
    if r is None:
        return
    buf = C.create_string_buffer(4096)
    assert r.ref_ledger_lookup(str(ledger).encode(), kml.encode(), HCS.encode(), buf, len(buf)) == 1
    c_ms, tm, tn, _ = buf.value.decode().split(" ", 3)
    assert (int(tm), int(tn)) == rows[0][4:6]
    other = '{"op":"reduce","dtype":"fp32","dims":[1048576]}'
    assert r.ref_ledger_commit(str(ledger).encode(), other.encode(), HCS.encode(), -1.0, 0.0) == 0
    rc, out = abi.run_kml(HCS, other, str(ledger))
    assert rc == 0 and "LEDGER HIT" in out, out
