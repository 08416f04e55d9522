"""Link-level drop-in: the reference's own apps, built from its unmodified sources by
local-ai-gpu-acceleration_b200/link/Makefile, with their hot decode launchers resolved to
libqgemv_b200.so.

CPU: every launcher the library exports is an undefined dynamic symbol of the apps that
call it (bound to the library at load time) and is local in the leftover reference
kernel object, so nothing is defined twice.
GPU: the apps run on packs written in the reference's manifest format and their own CPU
reference gate passes on this library's kernels (runtime_iq_matvec_probe,
runtime_q5k_matvec_probe, runtime_fused_bench --check-reference --check-only for the raw
and split Q4_K launchers, runtime_mixed_sequence_bench --check-reference).
"""

import json
import os
import subprocess
import sys

import pytest

from conftest import REPO

LINK = REPO / "local-ai-gpu-acceleration_b200" / "link"
BUILD = LINK / "_build"
APPS = ["mixed_sequence_benchmark_runner", "iq_matvec_probe", "q5k_matvec_probe",
        "fused_benchmark_runner"]


def _built() -> bool:
    return all((BUILD / a).exists() for a in APPS) and (BUILD / "replaced_symbols.txt").exists()


@pytest.fixture(scope="module")
def apps():
    if not _built():
        sys.path.insert(0, str(REPO / "oracle"))
        import qoracle

        if not (qoracle.REFERENCE_ROOT / "runtime").is_dir():
            pytest.skip("reference apps not built and the reference tree is not present")
        subprocess.run(["make", "-s", "-C", str(LINK), "-j8"], check=True)
    return {a: BUILD / a for a in APPS}


def _nm(path, *flags):
    out = subprocess.run(["nm", *flags, str(path)], capture_output=True, text=True, check=True).stdout
    return out.splitlines()


def test_apps_bind_the_hot_launchers_to_the_library(apps):
    replaced = set((BUILD / "replaced_symbols.txt").read_text().split())
    assert len(replaced) >= 20  # the Q4_K / Q5_K / IQ launchers, output sampler, feedback
    for name, path in apps.items():
        undefined = {l.split()[-1] for l in _nm(path, "-D", "--undefined-only") if "rtxllm_launch_" in l}
        defined_global = {l.split()[-1] for l in _nm(path) if " T rtxllm_launch_" in l}
        # every launcher the app needs from the replaced set comes from the library ...
        assert undefined and undefined <= replaced, (name, undefined - replaced)
        # ... and none of them is also defined globally inside the app
        assert not (defined_global & replaced), (name, defined_global & replaced)
    rest = {l.split()[-1] for l in _nm(BUILD / "decode_kernels_rest.o") if " T rtxllm_launch_" in l}
    assert not (rest & replaced)
    needed = subprocess.run(["readelf", "-d", str(apps["iq_matvec_probe"])], capture_output=True,
                            text=True, check=True).stdout
    assert "libqgemv_b200.so" in needed


# keys of the apps' JSON that explain a failed reference gate
_REFERENCE_KEYS = ("reference_passed", "reference_tolerance", "max_logit_abs_error",
                   "max_logit_error_row", "logit_mismatches", "kv_mismatches", "token_expected",
                   "token_observed", "reference_stage_mismatches", "reference_stage_results")


def _run(cmd, **kw) -> dict:
    res = subprocess.run([str(c) for c in cmd], capture_output=True, text=True, timeout=600, **kw)
    text = res.stdout
    try:
        out = json.loads(text[text.index("{"): text.rindex("}") + 1])
    except ValueError:
        out = None
    if res.returncode != 0:
        why = {k: out[k] for k in _REFERENCE_KEYS if out and k in out}
        raise AssertionError(f"rc {res.returncode}: {res.stderr[-1500:]} {json.dumps(why)[:6000]}")
    return out


@pytest.mark.gpu
@pytest.mark.parametrize("fmt_name", ["IQ2_S", "IQ3_S"])
def test_iq_matvec_probe_reference_gate(apps, tmp_path, fmt_name):
    from qgemv_b200 import manifest, packs

    fmt = manifest.FORMAT_OF_TYPE[fmt_name]
    name = "blk.0.ffn_gate.weight"
    pk = packs.synthetic_pack(fmt, 4096, 4096, seed=5 + fmt)
    m = manifest.write_raw_manifest(tmp_path, [(name, pk)])
    out = _run([apps["iq_matvec_probe"], "--iq-manifest", m, "--tensor", name,
                "--rows-limit", 512, "--steps", 4])
    assert out["reference_passed"] is True, out
    assert out["rows_checked"] == 512 and out["logit_mismatches"] == 0 and out["kv_mismatches"] == 0
    assert out["token_expected"] == out["token_observed"]


@pytest.mark.gpu
def test_q5k_matvec_probe_reference_gate(apps, tmp_path):
    from qgemv_b200 import manifest, packs

    name = "output.weight"
    pk = packs.synthetic_pack(packs.Q5K, 2048, 4096, seed=51)
    m = manifest.write_raw_manifest(tmp_path, [(name, pk)])
    out = _run([apps["q5k_matvec_probe"], "--q5k-manifest", m, "--tensor", name,
                "--rows-limit", 512, "--steps", 4])
    assert out["reference_passed"] is True, out


@pytest.mark.gpu
@pytest.mark.parametrize("kernel", ["direct", "vec4x4", "predecoded", "split-predecoded",
                                    "split-half", "split-compact", "split-native"])
def test_fused_runner_q4k_reference_gate(apps, tmp_path, kernel):
    from qgemv_b200 import manifest, packs

    rows, cols = 512, 4096
    pk = packs.synthetic_pack(packs.Q4K_RAW, rows, cols, seed=61)
    if kernel == "split-half":
        # The fp16 scale x min products of split-half are lossy and the runner's tolerance
        # for them is absolute (1.25e-2, fused_benchmark_runner/main.cpp:780), so this pack's
        # block scales are drawn 20x smaller than the BASELINE range to keep the format's own
        # rounding inside it (the reference's kernel rounds the same products).
        import numpy as np

        blk = pk.payload.reshape(-1, 144)
        rng = np.random.default_rng(62)
        scales = rng.uniform(5e-5, 5e-4, size=(blk.shape[0], 2)).astype(np.float16)
        blk[:, 0:4] = scales.view(np.uint8).reshape(-1, 4)
    blocks = tmp_path / "w.q4k_blocks.bin"
    blocks.write_bytes(pk.payload.tobytes())
    cmd = [apps["fused_benchmark_runner"], "--q4k-kernel", kernel, "--q4k-blocks-file", blocks,
           "--rows", rows, "--cols", cols, "--check-reference", "--check-only"]
    if kernel.startswith("split-"):
        payload, meta = packs.split_q4k(pk.payload, manifest.Q4K_POLICIES[kernel][0])
        (tmp_path / "p.bin").write_bytes(payload.tobytes())
        (tmp_path / "m.bin").write_bytes(meta.tobytes())
        cmd += ["--q4k-payload-file", tmp_path / "p.bin", "--q4k-meta-file", tmp_path / "m.bin"]
    out = _run(cmd)
    assert out["reference_checked"] is True and out["reference_passed"] is True, out


@pytest.mark.gpu
def test_mixed_runner_layer_sequence_reference_gate(apps, tmp_path):
    """The reference's mixed layer-sequence runner: Q4_K, IQ2_S, IQ3_S and Q5_K stages of one
    layer chained through its RMSNorm feedback, captured as one CUDA graph, every stage
    checked by its own CPU reference."""
    from qgemv_b200 import manifest, packs

    # source order: attention (q, k, v), then the FFN, then the output head
    iq_q = [("blk.0.attn_q.weight", packs.synthetic_pack(packs.IQ3S, 4096, 4096, seed=74))]
    q4k = [("blk.0.attn_k.weight", packs.synthetic_pack(packs.Q4K_RAW, 1024, 4096, seed=71)),
           ("blk.0.attn_v.weight", packs.synthetic_pack(packs.Q4K_RAW, 1024, 4096, seed=72))]
    iq_g = [("blk.0.ffn_gate.weight", packs.synthetic_pack(packs.IQ2S, 2048, 4096, seed=73))]
    q5 = [("output.weight", packs.synthetic_pack(packs.Q5K, 2048, 4096, seed=75))]
    # one source file's offsets for all five tensors (the runner orders stages by them)
    offs, at = [], 1 << 20
    for _, pk in iq_q + q4k + iq_g + q5:
        offs.append(at)
        at += (pk.payload.size + 31) // 32 * 32
    mq = manifest.write_q4k_manifest(tmp_path / "q4k", q4k, "split-native", source_offsets=offs[1:3])
    mi = manifest.write_raw_manifest(tmp_path / "iq", iq_q + iq_g, source_offsets=[offs[0], offs[3]])
    m5 = manifest.write_raw_manifest(tmp_path / "q5k", q5, source_offsets=offs[4:])
    out = _run([apps["mixed_sequence_benchmark_runner"], "--q4k-manifest", mq, "--iq-manifest", mi,
                "--q5k-manifest", m5, "--no-source-plan-validation", "--check-reference",
                "--rows-limit", 256, "--steps", 4])
    assert out.get("reference_passed") is True, json.dumps(out)[:3000]
