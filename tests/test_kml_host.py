"""The host side of the KML contract (CPU only, through the C ABI).

The declarations, ledger keys, canonical forms, workloads, exports and
rejection texts are pinned by tests/golden/kml_contract.json, which
tests/golden/make_golden.py produced by running the reference's own compiled
kml_import / canonical_form / op_signature / workload_of / hcs_fingerprint
(src/kml_front.cpp:75-251, src/kml.cpp:60-177, src/hcs.cpp:52-115,
src/main.cpp:217-219).  The tile plan and the runner's failure paths need no
GPU: with no device, a run must fail without touching the ledger (the
reference commits only a verified run, src/main.cpp:540-561).
"""
import json
from pathlib import Path

import pytest

import unikern_b200.abi as abi

GOLD = json.loads((Path(__file__).resolve().parent / "golden" / "kml_contract.json").read_text())
B200_HCS = (abi.SAMPLES / "hcs_nvidia_b200.json").read_text()


def gpu_present():
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.mark.parametrize("case", [c for c in GOLD["cases"] if c["rc"] == 0], ids=lambda c: c["canonical"][:40])
def test_contract_matches_reference(case):
    d = abi.kml_describe(case["kml"], GOLD["hcs_amd"], 148)
    assert d["canonical"] == case["canonical"]
    assert d["ledger_key"] == case["ledger_key"]
    assert int(d["ops"]) == case["ops"] and int(d["bytes"]) == case["bytes"]
    assert d["export"] == case["export"]


@pytest.mark.parametrize("case", [c for c in GOLD["cases"] if c["rc"] != 0], ids=lambda c: c["kml"][:40])
def test_rejections_match_reference(case):
    with pytest.raises(abi.UkError) as e:
        abi.kml_describe(case["kml"])
    assert e.value.code == 2
    assert str(e.value).split(": ", 1)[1] == case["error"]


def test_export_round_trips():
    for case in GOLD["cases"]:
        if case["rc"] == 0:
            d = abi.kml_describe(case["kml"])
            assert abi.kml_describe(d["export"])["canonical"] == d["canonical"]


def test_tolerance_table():
    for dt, tol in GOLD["tolerance"].items():
        if dt == "int8":
            continue
        d = abi.kml_describe('{"op":"gemm","dtype":"%s","dims":[8,8,8]}' % dt)
        assert float(d["tolerance"]) == tol


def test_b200_hcs_parses_and_fingerprints_stably():
    a = abi.kml_describe('{"op":"gemm","dtype":"fp16","dims":[8192,8192,8192]}', B200_HCS)
    b = abi.kml_describe('{"op":"gemm","dtype":"fp16","dims":[8192,8192,8192]}', B200_HCS)
    assert a["hcs_fingerprint"] == b["hcs_fingerprint"] and len(a["hcs_fingerprint"]) == 16
    assert a["ledger_key"].startswith("gemm:fp16:8192x8192x8192|" + a["hcs_fingerprint"] + "|")
    assert a["gap"] == ""


def _hcs_with_vram(mib):
    h = json.loads(B200_HCS)
    for t in h["tiers"]:
        if t["name"] == "vram":
            t["bytes"] = mib << 20
    return json.dumps(h)


def test_streamed_fp32_picks_the_tensor_core_ring_when_it_fits():
    # fp32 blocks of >= 2^30 multiply-adds take the split-tf32 tensor cores,
    # whose ring also holds B^T's tf32 pairs; a tighter device tier falls
    # back to the smaller FFMA ring
    kml = '{"op":"gemm","dtype":"fp32","dims":[8192,1024,1024]}'
    roomy = abi.kml_describe(kml, _hcs_with_vram(64))["placement"]
    tight = abi.kml_describe(kml, _hcs_with_vram(40))["placement"]
    assert "placement: streamed" in roomy and "split-tf32 tensor cores" in roomy
    assert "placement: streamed" in tight and "FFMA" in tight


@pytest.mark.parametrize("kml,mib,want", [
    ('{"op":"gemm","dtype":"fp16","dims":[4096,1024,1024]}', 16, "streamed"),   # 18 MiB > 0.85 x 16
    ('{"op":"gemm","dtype":"fp16","dims":[1024,1024,1024]}', 16, "resident"),   # 6 MiB fits
    ('{"op":"gemm","dtype":"fp32","dims":[1024,4096,1024]}', 16, "refused"),    # B alone is 16 MiB
    ('{"op":"softmax","dtype":"fp32","dims":[8192,1024]}', 16, "refused"),     # only a gemm streams
    ('{"op":"gemm","dtype":"fp16","dims":[8192,8192,8192]}', 183359, "resident"),
])
def test_placement_resident_streamed_or_refused(kml, mib, want):
    # scenario B: a gemm beyond 0.85 x the device tier keeps B resident and
    # streams A / C through a ring of row blocks (multiples of 256 rows)
    d = abi.kml_describe(kml, _hcs_with_vram(mib))
    assert d["placement"].startswith("placement: " + want), d["placement"]
    if want == "streamed":
        assert "1280-row blocks" in d["placement"]


@pytest.mark.parametrize("kml,gap", [
    ('{"op":"reduce","dtype":"int8","dims":[4]}', "dtype=int8 for op=reduce"),
    ('{"op":"conv","dtype":"fp16","dims":[32,32,8,3,3,16]}', "needs C a multiple of 64"),
    ('{"op":"gemm","dtype":"int8","dims":[4,4,4]}', "dtype=int8"),
    ('{"op":"gemm","dtype":"fp32","dims":[4,4,4],"children":[{"op":"reduce","dtype":"fp32","dims":[8]}]}',
     "children"),
    ('{"op":"conv","dtype":"fp32","dims":[2,2,4,3,3,8]}', "filter larger"),
])
def test_capability_gaps(kml, gap):
    assert gap in abi.kml_describe(kml)["gap"]


# the plans the kernels launch, on a 148-SM B200 (the ledger's tm / tn)
@pytest.mark.parametrize("op,dims,f16,want", [
    ("gemm", (8192, 8192, 8192), True, (256, 256, 64, 6)),     # tcgen05 SM-pair tile
    ("gemm", (128, 4096, 4096), True, (128, 256, 64, 4)),      # one 128-row block: single-SM tile
    ("gemm", (8192, 8192, 8190), True, (128, 128, 8, 2)),      # K % 8: CUDA-core path
    ("gemm", (512, 512, 512), False, (64, 64, 16, 2)),         # 64 tiles of 64x64, 8x8 per thread, K split 4
    ("gemm", (4096, 4096, 4096), False, (256, 256, 32, 3)),    # split-tf32 on the conv pair kernel
    ("gemm", (4096, 4096, 4090), False, (128, 128, 8, 2)),     # K % 32: FFMA
    ("conv", (58, 58, 256, 3, 3, 256), False, (256, 256, 32, 3)),
    ("conv", (58, 58, 256, 3, 3, 256), True, (256, 256, 64, 6)),
    ("conv", (32, 32, 8, 3, 3, 16), False, (64, 64, 8, 2)),     # C % 32: FFMA
    ("reduce", (134217728,), False, (1, 113360, 0, 1184)),     # 1184 splits = 8 CTAs/SM
    ("reduce", (4096,), False, (1, 4096, 0, 1)),
    ("softmax", (8192, 16384), False, (1, 16384, 0, 1)),
    ("rmsnorm", (8, 100000), False, (1, 2048, 0, 2)),          # streams twice
    ("channelscale", (65536, 256), False, (16, 256, 0, 1)),
    ("channelscale", (8192, 16384), False, (1, 16384, 0, 1)),   # long rows: one CTA per row
])
def test_tile_plan(op, dims, f16, want):
    assert abi.tile_plan(op, dims, f16, sms=148) == want


def test_solver_reports_the_plan_and_a_roofline_cost():
    d = abi.kml_describe('{"op":"gemm","dtype":"fp16","dims":[8192,8192,8192]}', B200_HCS, 148)
    assert d["tile"] == "256x256" and d["k_block"] == "64" and d["stages"] == "6"
    # 1.0995e12 flop at 2.25 PFLOP/s + 384 MiB over a 55 GB/s link
    assert float(d["c_ms"]) == pytest.approx(2 * 8192 ** 3 / 2.25e15 * 1e3 + 402653184 / 55e9 * 1e3, rel=1e-12)
    assert "tile=256x256" in d["placement"]


def test_run_without_a_device_commits_nothing(tmp_path):
    if gpu_present():
        pytest.skip("a GPU is present: the run would succeed")
    ledger = tmp_path / "ledger.jsonl"
    rc, out = abi.run_kml(B200_HCS, '{"op":"gemm","dtype":"fp32","dims":[64,64,64]}', str(ledger))
    assert rc == 1
    assert "RUN nvidia:cuda built=no ran=no verified=FAIL" in out
    assert "NOT committed" in out
    assert not ledger.exists() or ledger.read_text() == ""


def test_ledger_hit_reuses_the_recorded_tile(tmp_path):
    if gpu_present():
        pytest.skip("a GPU is present: covered by the GPU runner test")
    kml = '{"op":"softmax","dtype":"fp32","dims":[64,256]}'
    key = abi.kml_describe(kml, B200_HCS)["ledger_key"]
    ledger = tmp_path / "ledger.jsonl"
    row = "\t".join([key, "0.25", "0.5", "0.125", "1", "256", "placement: recorded"]) + "\n"
    ledger.write_text(row)
    rc, out = abi.run_kml(B200_HCS, kml, str(ledger))
    assert "LEDGER HIT  c_cached_ms=0.25  tile=1x256  (from ledger)" in out
    assert "placement: recorded" in out
    assert rc == 1 and ledger.read_text() == row


def test_bad_inputs_return_2():
    rc, out = abi.run_kml('{"vendor": "x"}', '{"op":"gemm","dtype":"fp32","dims":[4,4,4]}')
    assert rc == 2 and out.startswith("HCS missing required fields:")
    rc, out = abi.run_kml(B200_HCS, '{"op":"gemm","dtype":"fp32","dims":[4,4]}')
    assert rc == 2 and "rejected (1 violations)" in out
    rc, out = abi.run_kml(B200_HCS, '{"op":"conv","dtype":"fp16","dims":[32,32,8,3,3,16]}')
    assert rc == 2 and out.startswith("UNSUPPORTED: dtype=fp16 conv")


@pytest.mark.parametrize("kml", ['{"op":"softmax","dtype":"fp16","dims":[4,4]}',
                                 '{"op":"rmsnorm","dtype":"fp16","dims":[4,4]}',
                                 '{"op":"channelscale","dtype":"fp16","dims":[4,4]}',
                                 '{"op":"conv","dtype":"fp16","dims":[58,58,256,3,3,256]}'])
def test_fp16_widening_is_supported(kml):
    # the reference refuses these (src/codegen_hip.cpp:81-89); nvidia:cuda runs them
    assert abi.kml_describe(kml)["gap"] == ""
