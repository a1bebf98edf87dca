"""The ncu attribution report on CPU: both CSV shapes ncu writes (the long
--metrics form and the wide --page raw form with its units row), unit
normalisation, the reference's verdict rules (tools/summarize_ncu.py:105-117),
and the traffic / algorithmic-bytes ratio.  The inputs are small synthetic
captures written here."""
from __future__ import annotations

from pa_b200 import ncu_report as nr

_HEAD = ('"ID","Process ID","Process Name","Host Name","Kernel Name","Context","Stream",'
         '"Block Size","Grid Size","Device","CC","Section Name","Metric Name","Metric Unit",'
         '"Metric Value"')
_DEC = ('"0","1","python","h","void pa::decode::decode_kernel<__half, 64, 1>(pa::decode::Params)",'
        '"1","7","(416, 1, 1)","(148, 1, 1)","0","10.0","Command line profiler metrics",')
_EW = ('"1","1","python","h","at::native::vectorized_elementwise_kernel<4, float>(int)","1","7",'
       '"(128, 1, 1)","(1024, 1, 1)","0","10.0","Command line profiler metrics",')
LONG = "\n".join([
    "==PROF== Connected to process 123",
    _HEAD,
    _DEC + '"gpu__time_duration.sum","usecond","73.38"',
    _DEC + '"dram__bytes_read.sum","Mbyte","403.30"',
    _DEC + '"dram__bytes_write.sum","Mbyte","5.68"',
    _DEC + '"gpu__dram_throughput.avg.pct_of_peak_sustained_elapsed","%","68.1"',
    _DEC + '"sm__warps_active.avg.pct_of_peak_sustained_active","%","20.3"',
    _DEC + '"lts__t_sector_hit_rate.pct","%","0.45"',
    _EW + '"gpu__time_duration.sum","usecond","10.0"',
]) + "\n"

WIDE = "\n".join([
    '"ID","Process ID","Kernel Name","gpu__time_duration.sum","dram__bytes_read.sum",'
    '"dram__bytes_write.sum","dram__throughput.avg.pct_of_peak_sustained_elapsed",'
    '"sm__warps_active.avg.pct_of_peak_sustained_active","lts__t_sector_hit_rate.pct"',
    '"","","","ms","Gbyte","Mbyte","%","%","%"',
    '"0","9","prefill_tc_kernel<__nv_bfloat16, 128>","1.550","0.538","241.9","30.5","45.0","78.4"',
    '"1","9","prefill_tc_kernel<__nv_bfloat16, 128>","1.450","0.538","241.9","32.5","45.0","78.4"',
]) + "\n"


def test_long_form_and_units():
    recs = nr.parse(LONG)
    assert len(recs) == 2
    dec = next(r for r in recs if "decode_kernel" in r["kernel"])
    assert abs(dec["gpu__time_duration.sum"] - 73380.0) < 1e-6   # ns
    assert abs(dec["dram__bytes_read.sum"] - 403.30e6) < 1e-3     # bytes
    s = nr.summarize(recs, {"decode_kernel<__half, 64, 1>": 403_079_168}, peak_gbs=6531.3)
    e = s["decode_kernel<__half, 64, 1>"]
    assert e["launches"] == 1
    assert abs(e["traffic_bytes_per_launch"] - 408.98e6) < 1
    assert 1.0 < e["traffic_over_algorithmic"] < 1.02
    assert abs(e["achieved_gbs"] - 403_079_168 / 73380.0) < 1e-6
    assert 0.8 < e["frac_of_peak"] < 0.9
    # 68 % DRAM with 20 % occupancy: the reference's rules call it latency-bound
    assert e["verdict"].startswith("latency-bound")
    assert abs(e["share"] - 73.38 / 83.38) < 1e-9
    assert s["vectorized_elementwise_kernel<4, float>"]["verdict"] == "insufficient metrics"


def test_wide_form_with_units_row():
    recs = nr.parse(WIDE)
    assert len(recs) == 2
    assert abs(recs[0]["gpu__time_duration.sum"] - 1.55e6) < 1e-6
    assert abs(recs[0]["dram__bytes_read.sum"] - 0.538e9) < 1e-3
    assert abs(recs[0]["dram__bytes_write.sum"] - 241.9e6) < 1e-3
    s = nr.summarize(recs, 268e6)
    e = s["prefill_tc_kernel<__nv_bfloat16, 128>"]
    assert e["launches"] == 2 and abs(e["metrics"]["gpu__time_duration.sum"] - 1.5e6) < 1e-6
    assert e["verdict"].startswith("served from L2 (78% hits)")
    assert "re-reads" in e["verdict"]  # 780 MB of traffic for 268 MB


def test_verdict_rules():
    assert nr.verdict(75, 10, 90).startswith("bandwidth-bound")
    assert nr.verdict(50, 20, 90).startswith("latency-bound")
    assert nr.verdict(50, 40, 61).startswith("served from L2")
    assert nr.verdict(50, 40, 10).startswith("neither saturated")
    assert nr.verdict(None, 40, 10) == "insufficient metrics"


def test_cli(tmp_path, capsys):
    f = tmp_path / "cap.csv"
    f.write_text(LONG)
    assert nr.main([str(f), "--bytes-per-launch", "403079168", "--peak-gbs", "6531.3"]) == 0
    out = capsys.readouterr().out
    assert "decode_kernel<__half, 64, 1>" in out and "latency-bound" in out
    assert nr.main([str(f), "--json"]) == 0
    g = tmp_path / "empty.csv"
    g.write_text("==PROF== nothing\n")
    assert nr.main([str(g)]) == 1
