"""Host-side pieces of bench.py on CPU: the ncu CSV traffic reader, the
algorithmic byte count, the configuration record and the argument checks.
The timed paths need a B200 and run in the GPU suite's bench invocations."""

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

import bench  # noqa: E402
from blocksparsefa_reorder_b200 import workloads as W  # noqa: E402


def test_ncu_csv_traffic_reads_the_attention_launch(tmp_path):
    csv = tmp_path / "raw.csv"
    csv.write_text(
        '"ID","Kernel Name","dram__bytes_read.sum","dram__bytes_write.sum"\n'
        '"","","Mbyte","Kbyte"\n'
        '"0","plan_small_kernel","1.5","2"\n'
        '"1","void bsa::attn_tcp_kernel<128, 128, 1, 0>(...)","201.5","48500"\n')
    assert bench.ncu_csv_traffic(str(csv)) == pytest.approx(201.5e6 + 48.5e6)


def test_algorithmic_bytes_counts_q_o_and_each_heads_kv_once():
    wl = W.make("headline")
    units = wl.B * wl.H
    per_tensor = wl.N * wl.D * 2  # bf16 rows of one (b, h)
    # Q read + O written per unit, K and V of every key block some row keeps
    kept_cols = int(wl.mask.any(axis=0).sum())
    expect = units * (2 * per_tensor + 2 * kept_cols * wl.block * wl.D * 2)
    got = bench.algorithmic_bytes(wl, units)
    assert got == pytest.approx(expect, rel=0.02)


def test_config_dict_names_the_workload_and_its_shape():
    wl = W.make("sweep_p20")
    cfg = bench.config_dict(wl, 1, "weak")
    assert cfg["workload"].startswith("sweep_p20")
    assert (cfg["B"], cfg["H"], cfg["N"], cfg["D"], cfg["block"]) == (4, 32, 32768, 128, 64)
    assert cfg["dtype"] == "fp16" and abs(cfg["density"] - wl.density) < 1e-3


def test_scaling_and_warmup_rules():
    assert bench.scaling_of(1, "strong") == "weak"  # one GPU: nothing to split
    assert bench.scaling_of(8, "strong") == "strong"
    assert bench.scaling_of(8, "weak") == "weak"
    with pytest.raises(SystemExit):
        bench.main(["--warmup", "2"])
