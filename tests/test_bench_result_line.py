"""bench.py's RESULT line parses with the reference runner's regex
(scripts/run_bench_qwen_32b_fp16.sh:215-219, restated here as the interface
the line must keep), for sparse and dense tags."""
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
    line = bench.result_line(512, "32:64", "persistent", 50, 1000, 2.1735)
    ctx, tag, dtype, mode, med, mean, sd = REF_RESULT.findall(line)[-1]
    assert (ctx, tag, dtype, mode) == ("512", "M=64(32:64)", "float16", "b200_persistent")
    assert float(med) == float(mean) == 2.1735 and float(sd) == 0.0
    dense = bench.result_line(512, "dense", "persistent", 3, 10, 3.3)
    assert REF_RESULT.findall(dense)[-1][1] == "dense_float16"
