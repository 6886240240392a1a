"""bench.py's output contract and helpers, on the CPU: the reference arm
prints exactly one JSON line with the keys the driver reads, the clock
sampler turns nvidia-smi samples into the clocks record, and the synthetic
safetensors writer agrees with the loader's header parser."""
import json
import os
import pathlib
import subprocess
import sys

import numpy as np

ROOT = pathlib.Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))


def test_reference_arm_prints_one_json_line():
    env = dict(os.environ, RANK="0")
    out = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "1", "--warmup", "0",
                          "--dim", "64", "--codes", "256", "--levels", "2", "--cpu-rows", "32"],
                         capture_output=True, text=True, env=env, timeout=300, cwd=ROOT)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [ln for ln in out.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1, out.stdout
    line = json.loads(lines[0])
    for key in ("impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in line, key
    assert line["impl"] == "reference" and line["value"] > 0
    assert line["cpu_baseline"]["kind"] == "port" and line["cpu_baseline"]["cores"] >= 1
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["value"] == line["value"]


def test_non_zero_rank_of_the_reference_arm_prints_nothing():
    env = dict(os.environ, RANK="1")
    out = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "1", "--warmup", "0",
                          "--dim", "64", "--codes", "256", "--levels", "2", "--cpu-rows", "32"],
                         capture_output=True, text=True, env=env, timeout=300, cwd=ROOT)
    assert out.returncode == 0 and out.stdout.strip() == ""


class _FakeProc:
    def terminate(self):
        pass

    def wait(self, timeout=None):
        return 0


def test_clock_sampler_summarises_samples(tmp_path):
    import bench
    s = bench.ClockSampler(0)
    s.path = tmp_path / "clocks.csv"
    s.path.write_text(
        "0, 1400, 1965, 980.1, 0x4, Not Active, Not Active, Not Active, Active\n"
        "1, 1965, 1965, 300.0, 0x0, Not Active, Not Active, Not Active, Not Active\n"   # another GPU: ignored
        "0, 1380, 1965, 990.5, 0x4, Not Active, Not Active, Not Active, Active\n"
        "0, 1420, 1965, 995.0, 0x4, Not Active, Not Active, Not Active, Active\n")
    s.proc = _FakeProc()
    s.fh = open(tmp_path / "unused", "w")
    rec = s.stop()
    assert rec == {"sm_mhz": 1400.0, "sm_max_mhz": 1965.0, "samples": 3, "reasons": ["sw_power_cap"]}


def test_synthetic_checkpoint_writer_matches_the_header_parser(tmp_path):
    import bench
    from ncmorph_b200 import loader
    rng = np.random.default_rng(0)
    tensors = {"a": ("BF16", rng.integers(0, 1 << 16, (3, 5), dtype=np.uint16)),
               "b": ("F16", rng.standard_normal((7,)).astype(np.float16)),
               "c": ("F32", rng.standard_normal((2, 2, 3)).astype(np.float32))}
    path = tmp_path / "w.safetensors"
    total = bench._write_safetensors(path, tensors)
    assert path.stat().st_size == total
    h = loader.parse_header(path)
    raw = path.read_bytes()
    for name, (dtype, arr) in tensors.items():
        t = h.tensors[name]
        assert t.dtype == dtype and tuple(t.shape) == arr.shape
        off = h.offset(t)
        assert raw[off:off + t.data_end - t.data_begin] == arr.tobytes()
