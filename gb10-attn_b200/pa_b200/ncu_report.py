"""Attribution of a bandwidth result from an Nsight Compute capture.

The reference turns ncu's CSV into per-kernel means of a handful of counters
and one interpretive line (``tools/summarize_ncu.py:30-119``): DRAM
throughput above 70 % of peak is "bandwidth-bound", occupancy below 30 % with
DRAM below that is "latency-bound", an L2 hit rate above 60 % means the number
is not a DRAM measurement, anything else "neither saturated".  This module
applies the same rules to the B200 captures and adds what the reference left
to the reader: DRAM traffic per launch against the algorithmic bytes (re-reads
show as a ratio above 1) and, given the algorithmic bytes, the achieved rate
over the captured duration and its fraction of the measured copy peak.

It reads both CSV shapes ncu writes:

* long: ``ncu --csv --metrics ...`` (one row per launch and metric, columns
  "Kernel Name", "Metric Name", "Metric Unit", "Metric Value");
* wide: ``ncu -i report.ncu-rep --page raw --csv`` (one row per launch, one
  column per metric, a units row under the header).

``python -m pa_b200.ncu_report capture.csv [--bytes-per-launch N]
[--peak-gbs P] [--json]`` prints the summary; ``summarize`` returns it as a
dict for JSON results.
"""
from __future__ import annotations

import argparse
import csv
import io
import json
import re
import statistics
from collections import defaultdict
from pathlib import Path

# metric -> label; the reference's set plus the B200 captures' extras
METRICS = {
    "gpu__time_duration.sum": "duration",
    "dram__bytes_read.sum": "DRAM read",
    "dram__bytes_write.sum": "DRAM write",
    "dram__throughput.avg.pct_of_peak_sustained_elapsed": "DRAM %peak",
    "gpu__dram_throughput.avg.pct_of_peak_sustained_elapsed": "DRAM %peak",
    "lts__t_sector_hit_rate.pct": "L2 hit %",
    "l1tex__t_sector_hit_rate.pct": "L1 hit %",
    "sm__warps_active.avg.pct_of_peak_sustained_active": "occupancy %",
    "sm__throughput.avg.pct_of_peak_sustained_elapsed": "SM %peak",
    "smsp__issue_active.avg.pct_of_peak_sustained_active": "issue %",
    "sm__pipe_tensor_cycles_active.avg.pct_of_peak_sustained_active": "tensor pipe %",
    "launch__waves_per_multiprocessor": "waves/SM",
    "launch__registers_per_thread": "registers",
}
DRAM_PCT = ("dram__throughput.avg.pct_of_peak_sustained_elapsed",
            "gpu__dram_throughput.avg.pct_of_peak_sustained_elapsed")
OCCUPANCY = "sm__warps_active.avg.pct_of_peak_sustained_active"
L2_HIT = "lts__t_sector_hit_rate.pct"

_BYTES = {"byte": 1, "kbyte": 1e3, "mbyte": 1e6, "gbyte": 1e9, "tbyte": 1e12}
# the long form spells units out ("usecond"), the raw page abbreviates ("us")
_TIME_NS = {"nsecond": 1, "usecond": 1e3, "msecond": 1e6, "second": 1e9,
            "ns": 1, "us": 1e3, "ms": 1e6, "s": 1e9}


def _number(text: str) -> float | None:
    try:
        return float(str(text).replace(",", "").strip())
    except ValueError:
        return None


def _normalise(value: float, unit: str) -> float:
    """Bytes in bytes, durations in nanoseconds, everything else as given."""
    u = (unit or "").strip().lower()
    if u in _BYTES:
        return value * _BYTES[u]
    if u in _TIME_NS:
        return value * _TIME_NS[u]
    return value


def _table(text: str) -> list[list[str]]:
    lines = [ln for ln in text.splitlines() if ln.strip()]
    # banner lines (==PROF== ...) come before the header
    start = next((i for i, ln in enumerate(lines)
                  if ln.startswith('"ID"') or ln.startswith("ID,")), None)
    if start is None:
        return []
    return list(csv.reader(io.StringIO("\n".join(lines[start:]))))


def parse(source) -> list[dict]:
    """Launch records [{"kernel": name, "id": launch id, metric: value, ...}]
    from either CSV shape (a path, or the CSV text itself); values normalised
    (bytes, ns)."""
    if isinstance(source, Path) or (isinstance(source, str) and "\n" not in source):
        text = Path(source).read_text(errors="ignore")
    else:
        text = str(source)
    rows = _table(text)
    if not rows:
        return []
    head = rows[0]
    ix = {h: i for i, h in enumerate(head)}
    if "Kernel Name" not in ix:
        return []
    if "Metric Name" in ix:  # long form
        launches: dict[tuple, dict] = {}
        for r in rows[1:]:
            if len(r) < len(head):
                continue
            metric = r[ix["Metric Name"]]
            v = _number(r[ix["Metric Value"]]) if metric in METRICS else None
            if v is None:
                continue
            lid = r[ix["ID"]] if "ID" in ix else str(len(launches))
            key = (lid, r[ix["Kernel Name"]])
            rec = launches.setdefault(key, {"id": lid, "kernel": key[1]})
            unit = r[ix["Metric Unit"]] if "Metric Unit" in ix else ""
            rec[metric] = _normalise(v, unit)
        return list(launches.values())
    # wide form: header, a units row, then one row per launch
    body = rows[1:]
    units = {}
    if body and "ID" in ix and _number(body[0][ix["ID"]]) is None:
        units = {h: body[0][i] for h, i in ix.items() if i < len(body[0])}
        body = body[1:]
    out = []
    for r in body:
        if len(r) < len(head):
            continue
        rec = {"id": r[ix["ID"]] if "ID" in ix else str(len(out)),
               "kernel": r[ix["Kernel Name"]]}
        for metric in METRICS:
            if metric in ix:
                v = _number(r[ix[metric]])
                if v is not None:
                    rec[metric] = _normalise(v, units.get(metric, ""))
        out.append(rec)
    return out


def short_name(kernel: str) -> str:
    """void pa::decode::decode_kernel<__half, 64, 1>(...) -> decode_kernel<__half, 64, 1>."""
    k = re.sub(r"\(.*$", "", kernel or "").strip()
    k = re.sub(r"^(void\s+)?([\w:]+::)?", "", k)
    return k[:80] or "?"


def verdict(dram_pct: float | None, occupancy: float | None, l2_hit: float | None) -> str:
    """The reference's interpretive rule (tools/summarize_ncu.py:105-117)."""
    if dram_pct is None or occupancy is None:
        return "insufficient metrics"
    if dram_pct > 70:
        return "bandwidth-bound: near the bus, little left to win"
    if occupancy < 30:
        return "latency-bound: too few warps to cover DRAM latency"
    if l2_hit is not None and l2_hit > 60:
        return f"served from L2 ({l2_hit:.0f}% hits) -- not a DRAM measurement"
    return "neither saturated: check launch config / divergence"


def summarize(records: list[dict], bytes_per_launch: dict | float | None = None,
              peak_gbs: float | None = None) -> dict:
    """Per kernel: launch count, mean of every metric, share of the captured
    time, DRAM traffic per launch and its ratio to the algorithmic bytes (a
    number, or {short name: bytes}), the achieved GB/s of algorithmic bytes
    over the captured duration and its fraction of `peak_gbs`, and the verdict."""
    by: dict[str, list[dict]] = defaultdict(list)
    for r in records:
        by[short_name(r["kernel"])].append(r)
    total_ns = sum(r.get("gpu__time_duration.sum", 0.0) for r in records)
    out = {}
    for k, recs in by.items():
        means = {}
        for metric in METRICS:
            vals = [r[metric] for r in recs if metric in r]
            if vals:
                means[metric] = statistics.fmean(vals)
        ent = {"launches": len(recs), "metrics": means}
        dur = means.get("gpu__time_duration.sum")
        if dur is not None:
            ent["total_ns"] = sum(r.get("gpu__time_duration.sum", 0.0) for r in recs)
            ent["share"] = ent["total_ns"] / total_ns if total_ns else None
        rd, wr = means.get("dram__bytes_read.sum"), means.get("dram__bytes_write.sum")
        if rd is not None and wr is not None:
            ent["traffic_bytes_per_launch"] = rd + wr
        alg = bytes_per_launch.get(k) if isinstance(bytes_per_launch, dict) else bytes_per_launch
        if alg:
            ent["algorithmic_bytes_per_launch"] = alg
            if "traffic_bytes_per_launch" in ent:
                ent["traffic_over_algorithmic"] = ent["traffic_bytes_per_launch"] / alg
            if dur:
                ent["achieved_gbs"] = alg / dur  # bytes / ns = GB/s
                if peak_gbs:
                    ent["frac_of_peak"] = ent["achieved_gbs"] / peak_gbs
        dram = next((means[m] for m in DRAM_PCT if m in means), None)
        ent["verdict"] = verdict(dram, means.get(OCCUPANCY), means.get(L2_HIT))
        if ent.get("traffic_over_algorithmic", 1.0) > 1.10:
            ent["verdict"] += (f"; DRAM traffic {ent['traffic_over_algorithmic']:.2f}x the "
                               "algorithmic bytes: re-reads")
        out[k] = ent
    return out


def format_text(summary: dict) -> str:
    lines = []
    for k, e in sorted(summary.items(), key=lambda kv: -kv[1].get("total_ns", 0.0)):
        share = e.get("share")
        lines.append(f"{k}  ({e['launches']} launches"
                     + (f", {100 * share:.1f} % of captured time" if share is not None else "")
                     + ")")
        for metric, label in METRICS.items():
            if metric not in e["metrics"]:
                continue
            v = e["metrics"][metric]
            if "bytes" in metric:
                lines.append(f"    {label:14s} {v / 1e6:12.2f} MB")
            elif metric == "gpu__time_duration.sum":
                lines.append(f"    {label:14s} {v / 1e3:12.2f} us")
            else:
                lines.append(f"    {label:14s} {v:12.2f}")
        if "traffic_over_algorithmic" in e:
            lines.append(f"    traffic/alg    {e['traffic_over_algorithmic']:12.3f}")
        if "frac_of_peak" in e:
            lines.append(f"    achieved       {e['achieved_gbs']:12.1f} GB/s "
                         f"({100 * e['frac_of_peak']:.1f} % of peak)")
        lines.append(f"    -> {e['verdict']}")
    return "\n".join(lines)


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description="Attribution of an ncu capture (CSV).")
    ap.add_argument("csv")
    ap.add_argument("--bytes-per-launch", type=float, default=None)
    ap.add_argument("--peak-gbs", type=float, default=None)
    ap.add_argument("--json", action="store_true")
    a = ap.parse_args(argv)
    recs = parse(Path(a.csv))
    if not recs:
        print(f"{a.csv}: no parseable launches (profiling likely failed)")
        return 1
    s = summarize(recs, a.bytes_per_launch, a.peak_gbs)
    print(json.dumps(s, indent=1) if a.json else format_text(s))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
