"""Summarise an ncu report or launch-list CSV into the text kept in profiles/.

    python -m nkipy_b200.ncu_summary report <file.ncu-rep>
    python -m nkipy_b200.ncu_summary launches <launches.csv>
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
    """Per kernel: launches, total device time and share; when the capture also
    holds dram__bytes_{read,write}.sum, the mean DRAM bytes per launch, and a
    ``dram_bytes_per_launch`` line for the kernel with the largest share."""
    text = open(path).read()
    start = text.find('"ID"')
    rows = list(csv.reader(io.StringIO(text[start:])))
    hdr = rows[0]
    ii, ki = hdr.index("ID"), hdr.index("Kernel Name")
    mi, vi, ui = hdr.index("Metric Name"), hdr.index("Metric Value"), hdr.index("Metric Unit")
    tscale = {"ns": 1e-3, "nsecond": 1e-3, "us": 1.0, "usecond": 1.0, "ms": 1e3, "msecond": 1e3}
    bscale = {"byte": 1, "Kbyte": 1e3, "Mbyte": 1e6, "Gbyte": 1e9}
    per_launch = OrderedDict()  # launch id -> [name, us, dram bytes or None]
    for r in rows[1:]:
        if len(r) <= vi:
            continue
        rec = per_launch.setdefault(r[ii], [r[ki].split("(")[0], 0.0, None])
        v = float(r[vi].replace(",", ""))
        if r[mi] == "gpu__time_duration.sum":
            rec[1] += v * tscale.get(r[ui], 1.0)
        elif r[mi] in ("dram__bytes_read.sum", "dram__bytes_write.sum"):
            rec[2] = (rec[2] or 0.0) + v * bscale.get(r[ui], 1)
    agg = OrderedDict()
    for name, us, dram in per_launch.values():
        n, t, d = agg.get(name, (0, 0.0, None))
        agg[name] = (n + 1, t + us, d if dram is None else (d or 0.0) + dram)
    total = sum(t for _, t, _ in agg.values())
    has_dram = any(d is not None for _, _, d in agg.values())
    print(f"{'kernel':<60} {'launches':>8} {'total_us':>12} {'share':>7}" + (f" {'MB/launch':>10}" if has_dram else ""))
    ranked = sorted(agg.items(), key=lambda kv: -kv[1][1])
    for name, (n, t, d) in ranked:
        extra = f" {d / n / 1e6:>10.1f}" if has_dram and d is not None else ""
        print(f"{name[:60]:<60} {n:>8} {t:>12.1f} {100 * t / total:>6.1f}%" + extra)
    if has_dram and ranked and ranked[0][1][2] is not None:
        n, _, d = ranked[0][1]
        print(f"dram_bytes_per_launch: {d / n:.0f}")


if __name__ == "__main__":
    {"report": report, "launches": launches}[sys.argv[1]](sys.argv[2])
