"""bench.py's reference arm on the host cores: one JSON line with the keys the benchmark contract names, printed by
rank 0 only (other ranks exit 0 without work). It runs the reference's CPU path (the dense PyTorch definition,
impl="reference": the unmodified reference module when it is installed under baseline/_ref, "kind": "reference",
else this repository's restatement, "kind": "port") on a small shape, so it needs no GPU."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _run(env_extra):
    env = dict(os.environ, **env_extra)
    cmd = [sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "1", "--warmup", "0",
           "--shape", "1,1,256,16"]
    return subprocess.run(cmd, capture_output=True, text=True, env=env, cwd=ROOT, timeout=300)


def test_reference_arm_prints_one_contract_line():
    r = _run({"RANK": "0", "WORLD_SIZE": "1"})
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1
    d = json.loads(lines[0])
    for key in ("impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference" and d["value"] > 0 and d["unit"] == "TFLOP/s"
    installed = os.path.exists(os.path.join(ROOT, "baseline", "_ref", "kernel.py"))
    assert d["cpu_baseline"]["kind"] == ("reference" if installed else "port")
    assert d["cpu_baseline"]["value"] == d["value"]
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0
    assert d["config"]["T"] == 256 and d["config"]["D"] == 16


def test_reference_arm_other_ranks_print_nothing():
    r = _run({"RANK": "1", "WORLD_SIZE": "2"})
    assert r.returncode == 0, r.stderr[-2000:]
    assert r.stdout.strip() == ""


def test_e2e_pieces_cover_every_head_once():
    """The pipelined end-to-end step's pieces: every (sequence, head) of the shard in exactly one piece, equal groups
    of heads, at least the asked-for number of pieces when there are several sequences."""
    sys.path.insert(0, ROOT)
    import bench
    for Bs, Hs, want in [(4, 12, 4), (4, 12, 8), (2, 12, 4), (1, 12, 4), (1, 6, 4), (1, 7, 4), (8, 12, 4), (3, 5, 8)]:
        pieces = bench.e2e_chunks(Bs, Hs, want)
        seen = [(b, h) for b, h0, h1 in pieces for h in range(h0, h1)]
        assert sorted(seen) == [(b, h) for b in range(Bs) for h in range(Hs)], (Bs, Hs, want)
        assert len({h1 - h0 for _, h0, h1 in pieces}) == 1
        if Bs > 1:
            assert len(pieces) >= min(want, Bs * Hs)
