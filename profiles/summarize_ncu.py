"""Summarise an ncu report or launch-list CSV into the text kept in profiles/.

    python profiles/summarize_ncu.py report <file.ncu-rep>
    python profiles/summarize_ncu.py launches <launches.csv>
"""
import csv
import io
import subprocess
import sys
from collections import OrderedDict

METRICS = [
    "gpu__time_duration.sum",
    "dram__bytes_read.sum",
    "dram__bytes_write.sum",
    "gpu__dram_throughput.avg.pct_of_peak_sustained_elapsed",
    "sm__pipe_tensor_cycles_active.avg.pct_of_peak_sustained_elapsed",
    "sm__throughput.avg.pct_of_peak_sustained_elapsed",
    "sm__warps_active.avg.pct_of_peak_sustained_active",
    "launch__registers_per_thread",
    "launch__grid_size",
    "launch__block_size",
]


def report(path):
    raw = subprocess.run(["ncu", "-i", path, "--page", "raw", "--csv"], capture_output=True, text=True).stdout
    rows = list(csv.reader(io.StringIO(raw)))
    hdr, units = rows[0], rows[1]
    for r in rows[2:]:
        print(f"kernel: {r[hdr.index('Kernel Name')]}")
        vals = {}
        for m in METRICS:
            if m in hdr:
                i = hdr.index(m)
                print(f"  {m}: {r[i]} {units[i]}")
                vals[m] = (r[i], units[i])
        scale = {"byte": 1, "Kbyte": 1e3, "Mbyte": 1e6, "Gbyte": 1e9}
        tot = 0.0
        for m in ("dram__bytes_read.sum", "dram__bytes_write.sum"):
            v, u = vals.get(m, ("0", "byte"))
            tot += float(v.replace(",", "")) * scale.get(u, 1)
        print(f"dram_bytes_per_launch: {tot:.0f}")


def launches(path):
    text = open(path).read()
    start = text.find('"ID"')
    rows = list(csv.reader(io.StringIO(text[start:])))
    hdr = rows[0]
    ki, mi, vi, ui = hdr.index("Kernel Name"), hdr.index("Metric Name"), hdr.index("Metric Value"), hdr.index("Metric Unit")
    agg = OrderedDict()
    for r in rows[1:]:
        if len(r) <= vi or r[mi] != "gpu__time_duration.sum":
            continue
        name = r[ki].split("(")[0]
        scale = {"ns": 1e-3, "nsecond": 1e-3, "us": 1.0, "usecond": 1.0, "ms": 1e3, "msecond": 1e3}.get(r[ui], 1.0)
        n, t = agg.get(name, (0, 0.0))
        agg[name] = (n + 1, t + float(r[vi].replace(",", "")) * scale)
    total = sum(t for _, t in agg.values())
    print(f"{'kernel':<60} {'launches':>8} {'total_us':>12} {'share':>7}")
    for name, (n, t) in sorted(agg.items(), key=lambda kv: -kv[1][1]):
        print(f"{name[:60]:<60} {n:>8} {t:>12.1f} {100 * t / total:>6.1f}%")


if __name__ == "__main__":
    {"report": report, "launches": launches}[sys.argv[1]](sys.argv[2])
