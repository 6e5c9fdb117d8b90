"""Generate tests/golden/reference_vectors.npz from the UNIKERN reference itself.

Run where the reference tree is present, named by $UK_REFERENCE_TREE (the
UNIKERN project root):  ``UK_REFERENCE_TREE=<tree> python tests/golden/make_golden.py``.

Every output below is computed by the reference's own code, compiled by
oracle/build.py straight from the reference sources:
  * ``ref_cpu_conv`` / ``ref_cpu_reduce`` / ``ref_cpu_reduce_blocked``
    -> src/reference.cpp:6-48
  * ``emit_*`` -> the CPU references the generator embeds in its programs
    (src/codegen_hip.cpp:1124-1132 gemm, :1999-2009 softmax, :2168-2178
    rmsnorm, :2339-2344 channelscale, :604-605/:2167/:2338 initialisers)
  * ``ledger_key`` / ``canonical`` / ``workload`` -> src/kml.cpp, src/hcs.cpp,
    src/main.cpp:217-219
Inputs are seeded numpy draws (seed per case, listed in ``SEEDS``).
The fixture lets the oracle be pinned on machines without the reference.
"""
from __future__ import annotations

import ctypes as C
import json
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

from oracle import build as obuild  # noqa: E402
from oracle import oracle as O  # noqa: E402

OUT = Path(__file__).resolve().parent / "reference_vectors.npz"
SEEDS = {"gemm": 11, "gemm_f16": 12, "conv": 13, "reduce": 14, "softmax": 15,
         "rmsnorm": 16, "channelscale": 17}

# KML declarations whose ledger keys / canonical forms / workloads are pinned
KML_CASES = [
    '{"op":"gemm","dtype":"fp32","dims":[512,512,512],"tile_m":64,"tile_n":128,"layout":"NT"}',
    '{"op":"gemm","dtype":"fp16","dims":[8192,8192,8192],"layout":"NT"}',
    '{"op":"conv","dtype":"fp32","dims":[58,58,256,3,3,256]}',
    '{"op":"reduce","dtype":"fp32","dims":[134217728]}',
    '{"op":"softmax","dtype":"fp32","dims":[8192,16384]}',
    '{"op":"rmsnorm","dtype":"fp32","dims":[8192,16384]}',
    '{"op":"channelscale","dtype":"fp32","dims":[65536,256]}',
    '{"op":"gemm","dtype":"fp32","dims":[64,64,64],"children":[{"op":"reduce","dtype":"fp32","dims":[4096]},{"op":"gemm","dtype":"fp32","dims":[8,8,8]}]}',
]
# declarations the reference rejects (message text pinned)
KML_BAD = [
    '{"op":"gemm","dtype":"fp32","dims":[512,512]}',
    '{"op":"gemm","dtype":"fp64","dims":[1,2,3]}',
    '{"op":"conv","dtype":"fp32","dims":[8,8,2,3,3,-1],"tilem":4}',
    '{"op":"reduce","dtype":"fp32","dims":[3000000000]}',
    '{"op":"gemm","dtype":"fp32","dims":[4,4,4],"layout":"TN"}',
    '{"dtype":"fp32","dims":[4]}',
]


def main():
    if not obuild.build_ref():
        raise SystemExit("reference tree not found; set UK_REFERENCE_TREE")
    obuild.build_oracle()
    ref, emit = O.ref(), O.emit()
    out = {}

    # initialisers, idx 0..4095
    idx = np.arange(4096)
    for k in ("A", "B", "X", "W", "S"):
        out["init" + k] = np.array([getattr(emit, "emit_init" + k)(int(i)) for i in idx], np.float32)

    rng = np.random.default_rng(SEEDS["gemm"])
    A = rng.uniform(-1, 1, (33, 29)).astype(np.float32)
    B = rng.uniform(-1, 1, (29, 47)).astype(np.float32)
    Cm = np.zeros((33, 47), np.float32)
    emit.emit_gemm_cpu_ref(A, B, Cm, 33, 47, 29)
    out.update(gemm_A=A, gemm_B=B, gemm_C=Cm)
    As = out["initA"][: 64 * 64].reshape(64, 64).copy()
    Bs = out["initB"][: 64 * 64].reshape(64, 64).copy()
    Cs = np.zeros((64, 64), np.float32)
    emit.emit_gemm_cpu_ref(As, Bs, Cs, 64, 64, 64)
    out.update(gemm_saw_C=Cs)

    rng = np.random.default_rng(SEEDS["gemm_f16"])
    Ah = O.f32_to_f16(rng.normal(0, 0.5, (31, 37)).astype(np.float32))
    Bh = O.f32_to_f16(rng.normal(0, 0.5, (37, 45)).astype(np.float32))
    Ch = np.zeros((31, 45), np.float32)
    emit.emit_gemm_f16_cpu_ref(O.f16_to_f32(Ah), O.f16_to_f32(Bh), Ch, 31, 45, 37)
    out.update(gemm_f16_A=Ah, gemm_f16_B=Bh, gemm_f16_C=Ch)

    rng = np.random.default_rng(SEEDS["conv"])
    H, W, Cc, Kh, Kw, Oc = 10, 9, 3, 3, 3, 4
    x = rng.uniform(0, 1, (H, W, Cc)).astype(np.float32)
    wt = rng.normal(0, 0.3, (Oc, Kh, Kw, Cc)).astype(np.float32)
    y = np.zeros(Oc * (H - Kh + 1) * (W - Kw + 1), np.float32)
    ref.ref_cpu_conv(x.reshape(-1), wt.reshape(-1), y, H, W, Cc, Kh, Kw, Oc)
    y2 = np.zeros_like(y)
    emit.emit_conv(x.reshape(-1), wt.reshape(-1), y2, H, W, Cc, Kh, Kw, Oc)
    assert np.array_equal(y, y2), "reference.cpp and the emitted conv reference disagree"
    out.update(conv_x=x, conv_w=wt, conv_y=y, conv_dims=np.array([H, W, Cc, Kh, Kw, Oc], np.int32))

    rng = np.random.default_rng(SEEDS["reduce"])
    r = rng.normal(0, 1, 10007).astype(np.float32)
    alt = np.where(np.arange(1 << 16) % 2 == 1, np.float32(1e-6), np.float32(1e6)).astype(np.float32)
    out.update(reduce_x=r, reduce_alt=alt,
               reduce_seq=np.array([ref.ref_cpu_reduce(r, r.size), ref.ref_cpu_reduce(alt, alt.size)], np.float32),
               reduce_blk=np.array([ref.ref_cpu_reduce_blocked(r, r.size, 1024),
                                    ref.ref_cpu_reduce_blocked(alt, alt.size, 1024),
                                    emit.emit_reduce(r, r.size)], np.float32))

    rng = np.random.default_rng(SEEDS["softmax"])
    X = rng.normal(0, 2, (7, 300)).astype(np.float32)
    Y = np.zeros_like(X)
    emit.emit_softmax(X, Y, 7, 300)
    out.update(softmax_X=X, softmax_Y=Y)

    rng = np.random.default_rng(SEEDS["rmsnorm"])
    X = rng.normal(0, 1, (5, 257)).astype(np.float32)
    Wg = rng.normal(1, 0.1, 257).astype(np.float32)
    Y = np.zeros_like(X)
    emit.emit_rmsnorm(X, Wg, Y, 5, 257)
    out.update(rmsnorm_X=X, rmsnorm_W=Wg, rmsnorm_Y=Y)

    rng = np.random.default_rng(SEEDS["channelscale"])
    X = rng.normal(0, 1, (6, 33)).astype(np.float32)
    S = rng.uniform(0.5, 1.5, 33).astype(np.float32)
    Y = np.zeros_like(X)
    emit.emit_channelscale(X, S, Y, 6, 33)
    out.update(channelscale_X=X, channelscale_S=S, channelscale_Y=Y)

    hcs = (obuild.reference_tree() / "samples" / "hcs_amd.json").read_text()
    kml = {"hcs_amd": hcs, "cases": []}
    for k in KML_CASES:
        rc, canon = O.ref_str(ref.ref_kml_check, k)
        _, key = O.ref_str(ref.ref_ledger_key, k, hcs)
        ops, byt = C.c_longlong(), C.c_longlong()
        ref.ref_workload(k.encode(), C.byref(ops), C.byref(byt))
        _, exported = O.ref_str(ref.ref_kml_export, k)
        kml["cases"].append({"kml": k, "rc": rc, "canonical": canon, "ledger_key": key,
                             "ops": ops.value, "bytes": byt.value, "export": exported})
    for k in KML_BAD:
        rc, msg = O.ref_str(ref.ref_kml_check, k)
        kml["cases"].append({"kml": k, "rc": rc, "error": msg})
    kml["tolerance"] = {"fp32": ref.ref_tolerance_for(0), "fp16": ref.ref_tolerance_for(1),
                        "int8": ref.ref_tolerance_for(2)}
    (OUT.parent / "kml_contract.json").write_text(json.dumps(kml, indent=1) + "\n")

    np.savez_compressed(OUT, **out)
    print("wrote", OUT, OUT.stat().st_size, "bytes;", OUT.parent / "kml_contract.json")


if __name__ == "__main__":
    main()
