# SPDX-License-Identifier: MIT
"""The benchmark CLI (rmsnorm.benchmarks.benchmark_rmsnorm): argument rules, presets,
row selection and the speed-up arithmetic on the host, and one tiny timed row on a GPU.
Mirrors what the reference's tests/test_benchmark_helpers.py pins for its CLI."""

from __future__ import annotations

import argparse

import pytest
import torch

from rmsnorm.benchmarks import benchmark_rmsnorm as cli


def _args(*argv):
    return cli.build_parser().parse_args(list(argv))


def test_presets_listing_has_the_reference_layout():
    text = cli.format_presets().splitlines()
    assert text[0] == "preset,mode,gate_dtypes,fail_ratio,rows,description"
    assert text[1].startswith("large-backward,backward,bfloat16|float16,1.01,32768x65536|16384x131072|8192x262144,")
    assert text[2].startswith("mid-backward,backward,bfloat16|float16,1.01,32768x16384,")


def test_row_selection_and_filters():
    assert cli.select_rows(None, None, None, None) == cli.MN_PAIRS
    assert cli.select_rows([32768], [4096], None, None) == [(32768, 4096)]
    assert cli.select_rows(None, None, [(8, 64), (16, 64)], None) == [(8, 64), (16, 64)]
    assert cli.select_rows(None, [131072], None, "large-backward") == [(16384, 131072)]
    with pytest.raises(ValueError):
        cli.select_rows([1], None, None, None)
    with pytest.raises(ValueError):
        cli.select_rows(None, None, [(8, 64)], "mid-backward")


@pytest.mark.parametrize("argv,message", [
    (["--gate", "all", "--dtype", "float16"], "--gate cannot be combined with --dtype"),
    (["--backward", "--residual"], "--residual is only supported for forward benchmarks"),
    (["--residual-out-dtype", "float32"], "--residual-out-dtype requires --residual"),
    (["--fail-ratio", "0"], "--fail-ratio must be positive"),
    (["--min-speedup", "-1"], "--min-speedup must be nonnegative"),
    (["--preset", "mid-backward"], "--preset mid-backward requires --backward"),
    (["--input-pool-size", "0"], "--input-pool-size must be positive"),
])
def test_argument_rules(argv, message):
    with pytest.raises(ValueError, match=message):
        cli.validate_args(_args(*argv))


def test_pair_parsing():
    assert _args("--pair", "8,64").pair == [(8, 64)]
    with pytest.raises(SystemExit):
        _args("--pair", "8x64")


def test_speedup_summary_and_thresholds():
    res = [(1, 1, 0.5), (1, 2, 2.0), (1, 3, None)]
    s = cli.summarize(res)
    assert s["count"] == 2 and s["min"] == pytest.approx(-0.5) and s["max"] == pytest.approx(1.0)
    assert s["geomean"] == pytest.approx(0.0)
    assert cli.summarize([(1, 1, None)]) is None
    cli.check_thresholds([(1, 1, 0.99)], fail_ratio=1.01)
    with pytest.raises(ValueError, match="ratio threshold exceeded: 1x1=1.0200"):
        cli.check_thresholds([(1, 1, 1.02)], fail_ratio=1.01)
    with pytest.raises(ValueError, match="speedup threshold not met"):
        cli.check_thresholds([(1, 1, 0.95)], min_speedup=0.10)
    with pytest.raises(ValueError, match="no comparable rows"):
        cli.check_thresholds([(1, 1, None)], fail_ratio=1.0)


def test_list_presets_main(capsys):
    cli.main(["--list-presets"])
    assert capsys.readouterr().out.startswith("preset,mode,gate_dtypes")


@pytest.mark.gpu
@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device")
@pytest.mark.parametrize("extra", [[], ["--backward"], ["--residual", "--residual-out-dtype", "float32"]])
def test_one_small_row_on_the_gpu(tmp_path, extra):
    out = tmp_path / "rows.csv"
    cli.main(["--pair", "1024,2048", "--warmup", "2", "--rep", "5", "--input-pool-size", "2", "--summary",
              "--output", str(out), *extra])
    lines = out.read_text().splitlines()
    assert lines[0] == "M,N,pool_size,rmsnorm_ms,ref_ms,ratio,speedup,ref_config"
    row = lines[1].split(",")
    assert row[:2] == ["1024", "2048"] and float(row[3]) > 0 and float(row[4]) > 0
    assert lines[2].startswith("summary,count") and lines[3].startswith("summary,1,")
