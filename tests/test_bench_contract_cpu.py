"""bench.py's reference arm on the CPU: exactly one JSON line on stdout with the contract's keys."""
import json
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent


def test_reference_arm_prints_one_contract_line():
    res = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "1",
                          "--warmup", "0", "--layers", "2"],
                         capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert res.returncode == 0, res.stderr[-2000:]
    lines = [l for l in res.stdout.splitlines() if l.strip()]
    assert len(lines) == 1, res.stdout
    d = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference" and d["value"] > 0
    assert d["cpu_baseline"]["kind"] in ("port", "reference") and d["cpu_baseline"]["cores"] >= 1
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0


def test_reference_and_cast_arms_share_one_config():
    import argparse
    import bench
    a = argparse.Namespace(layers=32)
    assert bench.bench_config(a, 1) == bench.bench_config(a, 1)
    assert bench.bench_config(a, 8)["global_batch"] == 512


def test_weak_scaling_batch_keeps_configuration_3_at_one_gpu():
    import bench
    from cast_b200 import workloads
    w1 = bench.rank_workload(0, 1)
    c3 = workloads.config(3)
    assert w1.S == c3.S and w1.N == c3.N and w1.ids() == list(range(64))
    shards = [bench.rank_workload(r, 4) for r in range(4)]
    assert all(s.B == 64 for s in shards)
    assert sorted(i for s in shards for i in s.ids()) == list(range(256))


def test_traffic_parser_reads_an_ncu_raw_csv(tmp_path):
    import bench
    f = tmp_path / "raw.csv"
    f.write_text(
        '"ID","Process ID","Process Name","Host Name","Kernel Name","Context","Stream","Block Size","Grid Size",'
        '"Device","CC","dram__bytes_read.sum","dram__bytes_write.sum"\n'
        '"","","","","","","","","","","","Gbyte","Mbyte"\n'
        '"0","1","python","h","void attn_tc_kernel<1>(AttnParams)","1","7","(384, 1, 1)","(2, 512, 1)","0","10.0",'
        '"1.5","50"\n'
        '"1","1","python","h","void other_kernel()","1","7","(1, 1, 1)","(1, 1, 1)","0","10.0","9","9"\n')
    assert bench._traffic_from_csv(str(f)) == 1.55e9
