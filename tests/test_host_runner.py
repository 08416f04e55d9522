"""tp_decode_host (local-ai-gpu-acceleration_b200/link/tp_decode_host.cpp): the native
decode runner on the reference's runtime core -- VramSuperallocator arenas,
decide_admission(Strict) per rank with the ranks agreeing, one CUDA graph per context
bucket (CudaGraphBucket) -- around the library's decoder.

CPU (no GPU is touched before admission): an over-budget rank makes every rank print the
rejection object and exit 2 (the bench contract); within budget every rank is admitted.
GPU: graphs replayed per context bucket for successive tokens, the position advanced on
the device, reproduce the eager host-position steps bit for bit (TP 1, and TP 2 where two
GPUs are present)."""

import json
import subprocess

import pytest
import torch

from conftest import REPO
from test_link_dropin import BUILD, LINK, _built

HOST = BUILD / "tp_decode_host"
SMALL = ["--layers", "2", "--hidden", "1024", "--q-heads", "8", "--kv-heads", "4", "--ffn", "2048",
         "--vocab", "1024", "--ctx-max", "256"]


@pytest.fixture(scope="module")
def host():
    if not (_built() and HOST.exists()):
        import sys

        sys.path.insert(0, str(REPO / "oracle"))
        import qoracle

        if not (qoracle.REFERENCE_ROOT / "runtime").is_dir():
            pytest.skip("runner not built and the reference tree is not present")
        subprocess.run(["make", "-s", "-C", str(LINK), "-j8"], check=True)
    return HOST


def _ranks(host, tp, rdv, extra, timeout=600):
    procs = [subprocess.Popen([str(host), "--tp", str(tp), "--rank", str(r), "--rendezvous", str(rdv),
                               *[str(e) for e in extra(r)]], stdout=subprocess.PIPE,
                              stderr=subprocess.PIPE, text=True) for r in range(tp)]
    out = []
    for p in procs:
        so, se = p.communicate(timeout=timeout)
        out.append((p.returncode, so, se))
    return out


def _json(text):
    return json.loads(text[text.index("{"): text.rindex("}") + 1])


@pytest.mark.parametrize("tp", [2, 4])
def test_admission_rejects_every_rank_when_one_is_over_budget(host, tmp_path, tp):
    """70B-class shards; the last rank sees 5 GB free (its shard needs more): all ranks exit 2
    with the rejection object naming that rank and its over-budget bytes."""
    last = tp - 1
    res = _ranks(host, tp, tmp_path, lambda r: ["--admission-only", "--vram-free-bytes",
                                                5_000_000_000 if r == last else 180_000_000_000])
    for r, (rc, so, se) in enumerate(res):
        assert rc == 2, (r, rc, se)
        j = _json(so)
        assert j["admitted"] is False and j["rejected_rank"] == last
        assert j["weight_bytes"] > 0 and j["graph_bytes"] > 0 and j["workspace_bytes"] > 0
        if r == last:
            assert j["over_budget_bytes"] > 0 and j["required_bytes"] > j["usable_bytes"]


def _reference_harness():
    """The reference's own bench harness module (tools/bench/native_harness.py), loaded
    from the reference tree when it is present."""
    import importlib.util
    import sys

    sys.path.insert(0, str(REPO / "oracle"))
    import qoracle

    path = qoracle.REFERENCE_ROOT / "tools" / "bench" / "native_harness.py"
    if not path.exists():
        pytest.skip("reference tree not present")
    spec = importlib.util.spec_from_file_location("native_harness", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_reference_harness_reads_the_runner(host, tmp_path):
    """The bench-harness contract through the reference's own harness code: run_command
    parses the runner's one JSON object and keeps its exit code (0 admitted, 2 rejected),
    and write_metric_artifact turns it into a harness row."""
    harness = _reference_harness()
    ok = harness.run_command([str(host), "--tp", "1", "--rank", "0", "--rendezvous", str(tmp_path / "a"),
                              "--admission-only", "--vram-free-bytes", "180000000000"], timeout=120)
    assert ok["returncode"] == 0 and "parse_error" not in ok
    assert ok["metrics"]["admitted"] is True and ok["metrics"]["required_bytes"] > 0
    bad = harness.run_command([str(host), "--tp", "1", "--rank", "0", "--rendezvous", str(tmp_path / "b"),
                               "--admission-only", "--vram-free-bytes", "5000000000"], timeout=120)
    assert bad["returncode"] == 2 and bad["metrics"]["admitted"] is False
    ok["name"] = "tp_decode_host"
    art = harness.write_metric_artifact(tmp_path, ok, stamp=1, generated_at="now")
    row = json.loads(art.read_text())
    assert row["returncode"] == 0 and row["admitted"] is True and row["command"][0] == str(host)


def test_admission_admits_within_budget(host, tmp_path):
    res = _ranks(host, 2, tmp_path, lambda r: ["--admission-only", "--vram-free-bytes", 180_000_000_000])
    for rc, so, se in res:
        assert rc == 0, se
        j = _json(so)
        assert j["admitted"] is True and j["required_bytes"] <= j["usable_bytes"]


@pytest.mark.gpu
@pytest.mark.parametrize("tp", [1, 2])
def test_bucket_graphs_replay_tokens_like_eager_steps(host, tmp_path, tp):
    if torch.cuda.device_count() < tp:
        pytest.skip(f"needs {tp} GPUs")
    res = _ranks(host, tp, tmp_path, lambda r: [*SMALL, "--ctx-buckets", "64,128,256",
                                                "--tokens", "150"])
    tokens = None
    for rc, so, se in res:
        assert rc == 0, (rc, se[-2000:], so[-2000:])
        j = _json(so)
        assert j["admitted"] is True and j["graph_matches_eager"] is True
        assert j["error_word"] == 0 and j["position_after"] == 150
        assert [b["replays"] for b in j["buckets"]] == [64, 64, 22]
        tokens = tokens or j["tokens_graph"]
        assert j["tokens_graph"] == tokens  # every rank holds the same tokens
