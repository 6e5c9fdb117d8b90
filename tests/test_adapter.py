"""The drop-in boundary as the reference's own types see it.

unikern_b200/adapter/runner_nvidia.cpp is the translation unit a maintainer
adds to the UNIKERN tree: `RunOutcome run_cuda(const Solution&, const Hcs&,
const KmlTree&, const std::string&)` (include/unikern/codegen.hpp:49-83,
:104-117) and `BackendNvidia : IBackend` (include/unikern/components.hpp:14-33).
Its check driver is compiled against the reference's unmodified headers and
linked with the reference compiled from its sources (oracle/_ref); it builds
trees with the reference's kml_import, solves with the reference's solve and
runs them through the adapter, as cmd_run's execute branch would
(src/main.cpp:416-436).
"""
import json
import subprocess

import pytest

import unikern_b200.abi as abi

HCS = (abi.SAMPLES / "hcs_nvidia_b200.json").read_text()


@pytest.fixture(scope="module")
def exe():
    from unikern_b200.adapter import build as ab
    path = ab.OUT / "adapter_check"
    try:
        built = ab.build()
    except RuntimeError as e:  # a broken adapter must fail the test, not skip it
        pytest.fail(str(e))
    if built is None and not path.exists():
        pytest.skip("adapter not built: needs the reference tree (UK_REFERENCE_TREE) and oracle/_ref")
    return path


def lines(exe, *args):
    r = subprocess.run([str(exe), *args], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr
    return [json.loads(x) for x in r.stdout.splitlines()]


def gpu_present():
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


def test_registry_appends_nvidia_after_the_reference_backends(exe):
    kmls = ['{"op":"gemm","dtype":"fp16","dims":[512,512,512]}', '{"op":"softmax","dtype":"fp32","dims":[64,1024]}',
            '{"op":"gemm","dtype":"int8","dims":[64,64,64]}', '{"op":"conv","dtype":"fp16","dims":[34,34,32,3,3,16]}']
    out = lines(exe, "backends", *kmls)
    reg = out[:4]
    assert [b["backend"] for b in reg] == ["amd:hip", "apple:metal", "intel:ocl", "nvidia:cuda"]
    assert [b["vendor"] for b in reg] == [0, 1, 2, 3]
    assert reg[3]["streaming"] is True
    gaps = {json.loads(g["kml"])["dtype"] + ":" + json.loads(g["kml"])["op"]: g["gaps"]["nvidia:cuda"]
            for g in out[4:]}
    # the backend's answer is the library's own (uk_kml_describe's gap)
    for g in out[4:]:
        assert g["gaps"]["nvidia:cuda"] == abi.kml_describe(g["kml"])["gap"]
    assert gaps["fp16:gemm"] == "" and gaps["fp32:softmax"] == ""
    assert "int8" in gaps["int8:gemm"]
    assert "C=32" in gaps["fp16:conv"]  # the fp16 conv steps 64 channels at a time


@pytest.mark.skipif(gpu_present(), reason="checks the no-device path")
def test_run_without_a_device_reports_it(exe):
    (r,) = lines(exe, "run", HCS, '{"op":"reduce","dtype":"fp32","dims":[4096]}')
    assert r["built"] == 0 and r["ran"] == 0 and r["exit_code"] == 4
    assert r["migrations"] == -1 and r["checks"] == -1  # no result line reached
    assert "no CUDA device" in r["log"]


TREES = [
    '{"op":"gemm","dtype":"fp32","dims":[512,512,512]}',
    '{"op":"gemm","dtype":"fp16","dims":[1024,1024,1024]}',
    '{"op":"conv","dtype":"fp32","dims":[34,34,32,3,3,16]}',
    '{"op":"reduce","dtype":"fp32","dims":[1048576]}',
    '{"op":"softmax","dtype":"fp32","dims":[256,4096]}',
    '{"op":"rmsnorm","dtype":"fp32","dims":[256,4096]}',
    '{"op":"channelscale","dtype":"fp32","dims":[256,4096]}',
]


@pytest.mark.gpu
def test_run_cuda_fills_the_reference_run_outcome(exe):
    for r in lines(exe, "run", HCS, *TREES):
        tree = json.loads(r["kml"])
        tol = 0.0625 if tree["dtype"] == "fp16" else 0.03125
        assert r["gap"] == ""
        assert (r["built"], r["ran"], r["verified"], r["exit_code"]) == (1, 1, 1, 0), r
        assert 0 <= r["max_rel"] <= tol
        assert r["measured_ms"] > 0 and 0 < r["kernel_ms"] <= r["measured_ms"]
        assert r["migrations"] == 0 and r["checks"] > 0
        assert 0 < r["vram_free"] <= r["vram_total"]
        assert r["stream_path"] == "pinned"
        assert "UNIKERN_RESULT backend=nvidia:cuda verify=PASS" in r["log"]
        assert "tile=%s" % r["tile"] in r["log"] or r["tile"]
