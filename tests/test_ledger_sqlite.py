"""The ledger record formats, CPU only, through `uk_solve_kml` (the nvidia
branch of `unikern solve`, src/main.cpp:276-343) and `uk_calibrate`.

A ledger path ending in ".jsonl" is the reference's TAB file ledger; every
other path (the reference's default is ledger.sqlite3) is an SQLite database
with the reference's tables (src/sqlite_ledger.cpp:44-66; the choice is
src/main.cpp:61-70).  Interop is checked against the reference's own ledger
code, compiled from its sources into oracle/_ref/libukref.so: a row this
library commits is a HIT for the reference's lookup with the same tile and
c_ms, and a row the reference commits is a HIT here and feeds calibration.
"""
import ctypes as C
import sqlite3

import pytest

import unikern_b200.abi as abi
from oracle import oracle as O

B200_HCS = (abi.SAMPLES / "hcs_nvidia_b200.json").read_text()
GEMM = '{"op":"gemm","dtype":"fp16","dims":[8192,8192,8192]}'
REDUCE = '{"op":"reduce","dtype":"fp32","dims":[134217728]}'
SCHEMA = {
    "solutions": ["key", "op_sig", "hcs_fp", "tree_hash", "c_ms", "measured_ms", "tm", "tn", "placement",
                  "kernel_ms"],
    "violations": ["id", "key", "rate", "threshold", "migrations", "checks", "vram_free", "ts"],
}


def ref_lookup(path, kml, hcs=B200_HCS):
    r = O.ref()
    buf = C.create_string_buffer(4096)
    rc = r.ref_ledger_lookup(str(path).encode(), kml.encode(), hcs.encode(), buf, len(buf))
    if rc != 1:
        return rc, None
    c_ms, tm, tn, placement = buf.value.decode().split(" ", 3)
    return rc, (float(c_ms), int(tm), int(tn), placement)


def test_solve_commits_a_reference_format_sqlite_row(tmp_path):
    path = tmp_path / "ledger.sqlite3"
    rc, out = abi.solve_kml(B200_HCS, GEMM, str(path))
    assert rc == 0 and out.startswith("SOLVED  x* tile="), out
    d = abi.kml_describe(GEMM, B200_HCS)
    with sqlite3.connect(path) as db:
        for table, cols in SCHEMA.items():
            assert [r[1] for r in db.execute("PRAGMA table_info(%s)" % table)] == cols
        rows = db.execute("SELECT key, op_sig, hcs_fp, tree_hash, c_ms, measured_ms, tm, tn, placement, kernel_ms "
                          "FROM solutions").fetchall()
    assert len(rows) == 1
    key, sig, fp, th, c_ms, measured, tm, tn, placement, kernel = rows[0]
    assert key == d["ledger_key"] == "%s|%s|%s" % (sig, fp, th)
    assert fp == d["hcs_fingerprint"] and sig == d["signature"]
    assert "%dx%d" % (tm, tn) == d["tile"] and placement == d["placement"]
    assert measured == c_ms and kernel == 0.0  # solve seeds measured_ms with c_ms
    # a second solve is a hit on the recorded tile
    rc, out = abi.solve_kml(B200_HCS, GEMM, str(path))
    assert rc == 0 and out.startswith("LEDGER HIT  c_cached_ms=") and "tile=%dx%d" % (tm, tn) in out


def test_jsonl_path_keeps_the_tab_file_ledger(tmp_path):
    path = tmp_path / "ledger.jsonl"
    rc, _ = abi.solve_kml(B200_HCS, REDUCE, str(path))
    assert rc == 0
    f = path.read_text().splitlines()[0].split("\t")
    assert len(f) == 7 and f[0] == abi.kml_describe(REDUCE, B200_HCS)["ledger_key"]


def test_no_ledger_write_when_asked(tmp_path):
    path = tmp_path / "ledger.sqlite3"
    rc, out = abi.solve_kml(B200_HCS, GEMM, str(path), write_ledger=False)
    assert rc == 0 and "SOLVED" in out
    with sqlite3.connect(path) as db:
        assert db.execute("SELECT count(*) FROM solutions").fetchone()[0] == 0


def test_unopenable_sqlite_path_is_refused(tmp_path):
    rc, out = abi.solve_kml(B200_HCS, GEMM, str(tmp_path / "missing_dir" / "ledger.sqlite3"))
    assert rc == 2 and out.startswith("LEDGER sqlite ledger open failed"), out


def test_unsupported_tree_writes_nothing(tmp_path):
    path = tmp_path / "ledger.sqlite3"
    rc, out = abi.solve_kml(B200_HCS, '{"op":"gemm","dtype":"int8","dims":[64,64,64]}', str(path))
    assert rc == 2 and out.startswith("UNSUPPORTED"), out
    assert not path.exists()


@pytest.mark.skipif(O.ref() is None, reason="reference-compiled ledger (oracle/_ref) not built")
@pytest.mark.parametrize("name", ["ledger.sqlite3", "ledger.jsonl"])
def test_our_row_is_a_hit_for_the_reference(tmp_path, name):
    path = tmp_path / name
    for kml in (GEMM, REDUCE):
        assert abi.solve_kml(B200_HCS, kml, str(path))[0] == 0
        rc, hit = ref_lookup(path, kml)
        assert rc == 1, "the reference's lookup missed our row"
        d = abi.kml_describe(kml, B200_HCS)
        assert "%dx%d" % hit[1:3] == d["tile"] and hit[3] == d["placement"]
        assert hit[0] == float(d["c_ms"])
    n_viol = C.c_int()
    assert O.ref().ref_ledger_counts(str(path).encode(), C.byref(n_viol)) == 2 and n_viol.value == 0


@pytest.mark.skipif(O.ref() is None, reason="reference-compiled ledger (oracle/_ref) not built")
@pytest.mark.parametrize("name", ["ledger.sqlite3", "ledger.jsonl"])
def test_reference_row_is_a_hit_here_and_calibrates(tmp_path, name):
    path = tmp_path / name
    r = O.ref()
    # the reference's solve-time row, then a run's row with measured timings
    assert r.ref_ledger_commit(str(path).encode(), GEMM.encode(), B200_HCS.encode(), -1.0, 0.0) == 0
    rc, hit = ref_lookup(path, GEMM)
    assert rc == 1
    rc, out = abi.solve_kml(B200_HCS, GEMM, str(path))
    assert rc == 0 and out.startswith("LEDGER HIT  c_cached_ms=") and "tile=%dx%d" % hit[1:3] in out, out
    # measured - kernel = 10 ms for the f16 gemm's 402,653,184 compulsory bytes
    assert r.ref_ledger_commit(str(path).encode(), GEMM.encode(), B200_HCS.encode(), 12.0, 2.0) == 0
    rc, cal, report = abi.calibrate(B200_HCS, str(path))
    assert rc == 0, report
    assert "usable_rows=1" in report and "link_bw_gbps" in cal
    bw = float(cal.split('"link_bw_gbps":')[1].split(",")[0].strip().strip("}"))
    assert abs(bw - 402653184 / 10e-3 / 1e9) < 1e-9 * bw
