"""bench.py keeps the reference benchmark's interface: its RESULT line parses
with the reference runner's regex (scripts/run_bench_qwen_32b_fp16.sh:215-219,
restated here as the interface the line must keep), and the reference's
environment (NM_M, CTX, BENCH_WARMUP, BENCH_REPEAT x BENCH_INNER;
benchmarks/bench_llama_3_8b_fp16_fixed_ptx.py:97-105) sets the defaults."""
import re

import bench

REF_RESULT = re.compile(
    r"^RESULT\s+CTX=(\d+)\s+(\S+)\s+dtype=(\S+)\s+"
    r"actual_mode=(\S+).*?decode_ms_per_token=([0-9.]+)"
    r"(?:\s+mean=([0-9.]+))?"
    r"(?:\s+stdev=([0-9.]+))?",
    flags=re.MULTILINE,
)


def test_result_line_parses_like_the_reference():
    st = {"median": 2.1735, "mean": 2.1741, "stdev": 0.0012, "repeat": 100, "inner": 10, "steps": 1000}
    line = bench.result_line(512, "32:64", "persistent", 50, st)
    ctx, tag, dtype, mode, med, mean, sd = REF_RESULT.findall(line)[-1]
    assert (ctx, tag, dtype, mode) == ("512", "M=64(32:64)", "float16", "b200_persistent")
    assert (float(med), float(mean), float(sd)) == (2.1735, 2.1741, 0.0012)
    assert "repeat=100" in line
    dense = bench.result_line(512, "dense", "persistent", 3, dict(st, repeat=1))
    assert REF_RESULT.findall(dense)[-1][1] == "dense_float16"


def test_reference_environment_sets_defaults(monkeypatch):
    import sys

    import pytest

    for k in ("NM_M", "CTX", "BENCH_WARMUP", "BENCH_REPEAT", "BENCH_INNER"):
        monkeypatch.delenv(k, raising=False)
    monkeypatch.setattr(sys, "argv", ["bench.py"])
    a = bench.parse_args()
    assert (a.nm, a.ctx, a.warmup, a.steps) == ("32:64", 512, 50, 1000)
    monkeypatch.setenv("NM_M", "16")
    monkeypatch.setenv("CTX", "256")
    monkeypatch.setenv("BENCH_WARMUP", "7")
    monkeypatch.setenv("BENCH_REPEAT", "5")
    a = bench.parse_args()
    assert (a.nm, a.ctx, a.warmup, a.steps, a.inner) == ("8:16", 256, 7, 50, 10)
    monkeypatch.setenv("BENCH_INNER", "4")
    a = bench.parse_args()
    assert (a.steps, a.inner) == (20, 4)
    monkeypatch.delenv("BENCH_INNER")
    monkeypatch.setattr(sys, "argv", ["bench.py", "--nm", "32:64", "--steps", "3"])
    a = bench.parse_args()
    assert (a.nm, a.steps) == ("32:64", 3)  # flags win
    monkeypatch.setenv("NM_M", "0")
    monkeypatch.setattr(sys, "argv", ["bench.py"])
    assert bench.parse_args().nm == "dense"
    monkeypatch.setenv("NM_M", "12")
    with pytest.raises(ValueError, match="Unsupported NM_M"):
        bench.parse_args()


def test_import_origin_guard(monkeypatch):
    """bench.py refuses a package or library from outside its own tree."""
    from pathlib import Path

    import pytest

    from spmv_decode_b200 import _lib

    bench.check_import_origin()
    monkeypatch.setattr(_lib, "LIB_PATH", Path("/opt/elsewhere/libnmsparse_b200.so"))
    with pytest.raises(RuntimeError, match="Foreign import"):
        bench.check_import_origin()
