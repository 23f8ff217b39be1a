"""Report over gemm_bench's bench.csv and bench.py's JSON lines: Markdown tables and SVG charts.

The reference turns results/bench.csv into charts plus a summary table (analysis/plot.py:1-48,
report.md). This module reads the same CSV schema (device,sm,M,N,K,kernel,ms,tflops,
pct_of_cublas,max_abs_err, src/main.cu:103; gemm_bench appends pct_of_peak,dtype, which older
files lack) and adds what the B200 build measures beside it: each row against the library
kernel of the same precision, and the GPU-count dimension from bench.py's JSON lines (one per
run, N = 1..8). With --charts DIR it also draws the reference's chart set per device - throughput
vs size, % of the same-precision library row vs size, throughput bars at the largest size, the
precision Pareto (error vs throughput) - plus throughput vs GPU count, as standalone SVG files
written by hand (no plotting library is needed).

    python report.py results/bench.csv [--bench-json runs.jsonl] [--out report.md] [--charts DIR]
"""
from __future__ import annotations

import argparse
import collections
import csv
import json
import math
import os

# same-precision library row for each of this repo's rows (and the reference's)
LIBRARY_OF = {
    "tc_f16": "cublas_tc", "ref_mma_warptile": "cublas_tc", "ref_wmma": "cublas_tc",
    "tc_fp8": "cublaslt_fp8", "ref_mma_fp8": "cublaslt_fp8", "tc_fp8_amax": "cublaslt_fp8_amax",
    "tc_mxfp4_b32": "cublaslt_mxfp4",
    # the reference's own rows (its analysis/plot.py uses cublas_tc as the FP16 ceiling)
    "wmma": "cublas_tc", "mma_base": "cublas_tc", "mma_swizzle": "cublas_tc", "mma_vec": "cublas_tc",
    "mma_pipe": "cublas_tc", "mma_warptile": "cublas_tc", "mma_fp8": "cublaslt_fp8",
}
ORDER = ["tc_f16", "tc_fp8", "tc_fp8_amax", "tc_fp4", "tc_fp4_amax", "tc_mxfp4", "tc_mxfp4_b32",
         "ref_wmma", "ref_mma_warptile", "ref_mma_fp8",
         "cublas", "cublas_tc", "cublaslt_fp8", "cublaslt_fp8_amax", "cublaslt_mxfp4"]


def load_csv(path: str) -> list[dict]:
    with open(path) as f:
        return list(csv.DictReader(f))


def load_json_lines(path: str) -> list[dict]:
    out = []
    with open(path) as f:
        for line in f:
            line = line.strip()
            if line.startswith("{"):
                out.append(json.loads(line))
    return out


def _rank(kernel: str) -> int:
    return ORDER.index(kernel) if kernel in ORDER else len(ORDER)


def size_tables(rows: list[dict]) -> list[str]:
    """One table per (device, problem size): throughput, % of the same-precision library row,
    % of the dtype's nominal dense peak, and the error the driver measured."""
    by = collections.defaultdict(dict)
    for r in rows:
        key = (r["device"], r["sm"], int(r["M"]), int(r["N"]), int(r["K"]))
        by[key][r["kernel"]] = r  # a later run of the same row replaces an earlier one
    lines = []
    for (dev, sm, M, N, K) in sorted(by, key=lambda k: (k[0], k[1], k[2] * k[3] * k[4], k[2])):
        kerns = by[(dev, sm, M, N, K)]
        lines += [f"### {dev} (sm_{sm}), M = {M}, N = {N}, K = {K}", "",
                  "| kernel | dtype | TFLOP/s | % of same-precision library | % of dense peak | max abs err |",
                  "|---|---|---|---|---|---|"]
        for k in sorted(kerns, key=lambda k: (_rank(k), k)):
            r = kerns[k]
            tf = float(r["tflops"])
            lib = LIBRARY_OF.get(k)
            pct = f"{100.0 * tf / float(kerns[lib]['tflops']):.1f}% of {lib}" if lib in kerns else "-"
            peak = f"{float(r['pct_of_peak']):.1f}%" if r.get("pct_of_peak") else "-"
            lines.append(f"| {k} | {r.get('dtype') or '-'} | {tf:.1f} | {pct} | {peak} | "
                         f"{float(r['max_abs_err']):.3g} |")
        lines.append("")
    return lines


def scaling_table(runs: list[dict]) -> list[str]:
    """bench.py lines grouped by workload: whole-box TFLOP/s per GPU count, the ratio to the
    one-GPU line of the same workload, and the gather columns when present."""
    groups = collections.defaultdict(list)
    for d in runs:
        if "unavailable" in d or d.get("impl", "ours") != "ours":
            continue
        groups[d.get("config", {}).get("workload", "?")].append(d)
    lines = []
    for wl in sorted(groups):
        ds = sorted(groups[wl], key=lambda d: d["n_gpus"])
        base = next((d["value"] for d in ds if d["n_gpus"] == 1), None)
        lines += [f"### {wl}", "",
                  "| GPUs | TFLOP/s (all GPUs) | x one GPU | ms per step | e2e TFLOP/s | NCCL gather ms | fused GEMM+gather ms |",
                  "|---|---|---|---|---|---|---|"]
        for d in ds:
            g = d.get("gather") or {}
            fused = g.get("fused") or {}
            ratio = f"{d['value'] / base:.2f}" if base else "-"
            e2e = (d.get("e2e") or {}).get("value", "-")
            lines.append(f"| {d['n_gpus']} | {d['value']:.1f} | {ratio} | {d['ms_per_step']} | {e2e} | "
                         f"{g.get('ms', '-')} | {fused.get('ms_per_step', '-')} |")
        lines.append("")
        sharded = [d for d in ds if d.get("sharded")]
        if sharded:
            lines += [f"#### {wl}: sharded record (strong scaling)", "",
                      "| GPUs | dtype | GEMM ms | GEMM TFLOP/s (all GPUs) | + NCCL gather ms | fused GEMM+gather ms | fused TFLOP/s |",
                      "|---|---|---|---|---|---|---|"]
            for d in sharded:
                for dt in ("f16", "fp8"):
                    r = d["sharded"].get(dt)
                    if not r:
                        continue
                    nc = (r.get("nccl_gather") or {}).get("gemm_plus_gather_ms", "-")
                    fu = r.get("fused_gather") or {}
                    lines.append(f"| {d['n_gpus']} | {dt} | {r['gemm_ms']} | {r['gemm_tflops_all_gpus']} | {nc} | "
                                 f"{fu.get('ms_per_step', '-')} | {fu.get('tflops_all_gpus', '-')} |")
            lines.append("")
    return lines


# ------------------------------------------------------------------ SVG charts
PALETTE = ["#1a73e8", "#d93025", "#188038", "#f9ab00", "#9334e6", "#12b5cb", "#e8710a", "#5f6368",
           "#b31412", "#0b8043", "#7a1fa2", "#174ea6", "#a50e0e", "#ea8600", "#3c4043"]
W, H, L, R, T, B = 760, 460, 70, 230, 50, 60  # canvas and margins (legend on the right)


def _esc(t: str) -> str:
    return str(t).replace("&", "&amp;").replace("<", "&lt;").replace(">", "&gt;")


def _ticks(lo: float, hi: float, n: int = 5) -> list[float]:
    if hi <= lo:
        hi = lo + 1.0
    step = 10 ** math.floor(math.log10((hi - lo) / n))
    for m in (1, 2, 5, 10):
        if (hi - lo) / (step * m) <= n:
            step *= m
            break
    t0 = math.floor(lo / step) * step
    return [t0 + i * step for i in range(int((hi - t0) / step) + 2) if t0 + i * step <= hi * 1.0001]


class Svg:
    """A minimal plotting canvas: one axes box, linear or log2/log10 x, linear y, a legend."""

    def __init__(self, title: str, xlabel: str, ylabel: str, xs: list[float], ys: list[float],
                 xlog: int = 0, ylo: float = 0.0):
        self.xlog = xlog
        fx = (lambda v: math.log(v, xlog)) if xlog else (lambda v: v)
        self.fx = fx
        lo, hi = min(fx(x) for x in xs), max(fx(x) for x in xs)
        if hi == lo:
            lo, hi = lo - 1, hi + 1
        pad = 0.05 * (hi - lo)
        self.x0, self.x1 = lo - pad, hi + pad
        self.y0, self.y1 = ylo, max(ys) * 1.12 if ys and max(ys) > 0 else 1.0
        self.parts = [f'<svg xmlns="http://www.w3.org/2000/svg" width="{W}" height="{H}" font-family="sans-serif" font-size="12">',
                      f'<rect width="{W}" height="{H}" fill="white"/>',
                      f'<text x="{(L + W - R) / 2}" y="24" text-anchor="middle" font-size="15">{_esc(title)}</text>',
                      f'<text x="{(L + W - R) / 2}" y="{H - 15}" text-anchor="middle">{_esc(xlabel)}</text>',
                      f'<text x="18" y="{(T + H - B) / 2}" text-anchor="middle" transform="rotate(-90 18 {(T + H - B) / 2})">{_esc(ylabel)}</text>',
                      f'<rect x="{L}" y="{T}" width="{W - L - R}" height="{H - T - B}" fill="none" stroke="#888"/>']
        for yv in _ticks(self.y0, self.y1):
            y = self.py(yv)
            self.parts.append(f'<line x1="{L}" y1="{y:.1f}" x2="{W - R}" y2="{y:.1f}" stroke="#e0e0e0"/>')
            self.parts.append(f'<text x="{L - 6}" y="{y + 4:.1f}" text-anchor="end">{yv:g}</text>')
        self.nleg = 0

    def px(self, x: float) -> float:
        return L + (self.fx(x) - self.x0) / (self.x1 - self.x0) * (W - L - R)

    def py(self, y: float) -> float:
        return H - B - (y - self.y0) / (self.y1 - self.y0) * (H - T - B)

    def xticks(self, values: list[float], labels: list[str] | None = None):
        for i, v in enumerate(values):
            x = self.px(v)
            lab = labels[i] if labels else f"{v:g}"
            self.parts.append(f'<line x1="{x:.1f}" y1="{H - B}" x2="{x:.1f}" y2="{H - B + 5}" stroke="#888"/>')
            self.parts.append(f'<text x="{x:.1f}" y="{H - B + 18}" text-anchor="middle">{_esc(lab)}</text>')

    def legend(self, label: str, color: str, dash: bool = False):
        y = T + 10 + 18 * self.nleg
        st = ' stroke-dasharray="5,3"' if dash else ""
        self.parts.append(f'<line x1="{W - R + 12}" y1="{y}" x2="{W - R + 32}" y2="{y}" stroke="{color}" stroke-width="3"{st}/>')
        self.parts.append(f'<text x="{W - R + 38}" y="{y + 4}">{_esc(label)}</text>')
        self.nleg += 1

    def line(self, pts: list[tuple[float, float]], color: str, label: str):
        pts = sorted(pts)
        d = " ".join(f"{self.px(x):.1f},{self.py(y):.1f}" for x, y in pts)
        self.parts.append(f'<polyline points="{d}" fill="none" stroke="{color}" stroke-width="2"/>')
        for x, y in pts:
            self.parts.append(f'<circle cx="{self.px(x):.1f}" cy="{self.py(y):.1f}" r="3.5" fill="{color}"/>')
        self.legend(label, color)

    def hline(self, y: float, color: str, label: str):
        self.parts.append(f'<line x1="{L}" y1="{self.py(y):.1f}" x2="{W - R}" y2="{self.py(y):.1f}" stroke="{color}" '
                          f'stroke-dasharray="5,3" stroke-width="1.5"/>')
        self.legend(label, color, dash=True)

    def point(self, x: float, y: float, color: str, label: str):
        self.parts.append(f'<circle cx="{self.px(x):.1f}" cy="{self.py(y):.1f}" r="6" fill="{color}"/>')
        self.parts.append(f'<text x="{self.px(x) + 9:.1f}" y="{self.py(y) - 6:.1f}">{y:.0f}</text>')
        self.legend(label, color)

    def text(self) -> str:
        return "\n".join(self.parts + ["</svg>"]) + "\n"


def bar_chart(title: str, ylabel: str, names: list[str], values: list[float]) -> str:
    n = max(1, len(values))
    ymax = max(values) * 1.15 if values and max(values) > 0 else 1.0
    bw = (W - L - 40) / n
    parts = [f'<svg xmlns="http://www.w3.org/2000/svg" width="{W}" height="{H}" font-family="sans-serif" font-size="12">',
             f'<rect width="{W}" height="{H}" fill="white"/>',
             f'<text x="{W / 2}" y="24" text-anchor="middle" font-size="15">{_esc(title)}</text>',
             f'<text x="18" y="{(T + H - B) / 2}" text-anchor="middle" transform="rotate(-90 18 {(T + H - B) / 2})">{_esc(ylabel)}</text>']
    for yv in _ticks(0.0, ymax):
        y = H - B - yv / ymax * (H - T - B)
        parts.append(f'<line x1="{L}" y1="{y:.1f}" x2="{W - 40}" y2="{y:.1f}" stroke="#e0e0e0"/>')
        parts.append(f'<text x="{L - 6}" y="{y + 4:.1f}" text-anchor="end">{yv:g}</text>')
    for i, (nm, v) in enumerate(zip(names, values)):
        x = L + i * bw + 0.15 * bw
        h = v / ymax * (H - T - B)
        parts.append(f'<rect x="{x:.1f}" y="{H - B - h:.1f}" width="{0.7 * bw:.1f}" height="{h:.1f}" fill="{PALETTE[i % len(PALETTE)]}"/>')
        parts.append(f'<text x="{x + 0.35 * bw:.1f}" y="{H - B - h - 4:.1f}" text-anchor="middle">{v:.0f}</text>')
        parts.append(f'<text x="{x + 0.35 * bw:.1f}" y="{H - B + 14}" text-anchor="end" '
                     f'transform="rotate(-30 {x + 0.35 * bw:.1f} {H - B + 14})" font-size="11">{_esc(nm)}</text>')
    return "\n".join(parts + ["</svg>"]) + "\n"


def device_charts(rows: list[dict], outdir: str) -> list[str]:
    """The reference's per-device chart set (analysis/plot.py:70-200) as SVG files in outdir;
    returns the Markdown lines that embed them. Square problems (M = N = K) only, as there."""
    by = collections.defaultdict(lambda: collections.defaultdict(dict))
    for r in rows:
        M, N, K = int(r["M"]), int(r["N"]), int(r["K"])
        if M == N == K:
            by[(r["device"], r["sm"])][r["kernel"]][M] = r
    md = []
    os.makedirs(outdir, exist_ok=True)
    for (dev, sm), kerns in sorted(by.items()):
        sizes = sorted({s for k in kerns.values() for s in k})
        names = sorted(kerns, key=lambda k: (_rank(k), k))
        color = {k: PALETTE[i % len(PALETTE)] for i, k in enumerate(names)}
        short = dev.replace("NVIDIA ", "")
        files = []
        tf_all = [float(r["tflops"]) for k in names for r in kerns[k].values()]
        # 1: throughput vs size
        c = Svg(f"GEMM throughput - {short} (sm_{sm})", "matrix size M = N = K", "TFLOP/s", sizes, tf_all, xlog=2)
        c.xticks(sizes)
        for k in names:
            c.line([(s, float(r["tflops"])) for s, r in kerns[k].items()], color[k], k)
        files.append((f"tflops_sm{sm}.svg", c.text(), "throughput vs size"))
        # 2: % of the same-precision library row
        pct = {}
        for k in names:
            lib = LIBRARY_OF.get(k)
            if lib in kerns:
                pts = [(s, 100.0 * float(r["tflops"]) / float(kerns[lib][s]["tflops"]))
                       for s, r in kerns[k].items() if s in kerns[lib] and float(kerns[lib][s]["tflops"]) > 0]
                if pts:
                    pct[k] = pts
        if pct:
            c = Svg(f"% of the same-precision library kernel - {short}", "matrix size M = N = K",
                    "% of library TFLOP/s", sizes, [y for p in pct.values() for _, y in p] + [100.0], xlog=2)
            c.xticks(sizes)
            for k, pts in pct.items():
                c.line(pts, color[k], f"{k} / {LIBRARY_OF[k]}")
            c.hline(100.0, "#188038", "library = 100%")
            files.append((f"pct_library_sm{sm}.svg", c.text(), "% of the same-precision library row"))
        # 3: bars at the largest size
        big = sizes[-1]
        present = [k for k in names if big in kerns[k]]
        files.append((f"bars_sm{sm}.svg",
                      bar_chart(f"Throughput at M = N = K = {big} - {short}", "TFLOP/s", present,
                                [float(kerns[k][big]["tflops"]) for k in present]), f"throughput bars at {big}"))
        # 4: precision Pareto at the largest size (error on a log10 axis)
        par = [(k, float(kerns[k][big]["max_abs_err"]), float(kerns[k][big]["tflops"])) for k in present
               if float(kerns[k][big]["max_abs_err"]) > 0]
        if len(par) >= 2:
            c = Svg(f"Precision Pareto at {big} - {short}", "max abs error (log scale, lower is better)",
                    "TFLOP/s", [e for _, e, _ in par], [t for _, _, t in par], xlog=10)
            ex = sorted({10.0 ** e for e in range(math.floor(math.log10(min(e for _, e, _ in par))),
                                                   math.ceil(math.log10(max(e for _, e, _ in par))) + 1)})
            c.xticks([e for e in ex if c.x0 <= math.log10(e) <= c.x1], None)
            for k, e, t in par:
                c.point(e, t, color[k], k)
            files.append((f"pareto_sm{sm}.svg", c.text(), "precision Pareto"))
        md += [f"### {dev} (sm_{sm})", ""]
        for fname, text, caption in files:
            with open(os.path.join(outdir, fname), "w") as f:
                f.write(text)
            md.append(f"![{caption}]({fname})")
        md.append("")
    return md


def scaling_chart(runs: list[dict], outdir: str) -> list[str]:
    """Whole-box TFLOP/s against GPU count: the headline per workload and, where present, the
    sharded record's GEMM alone and GEMM + fused gather, with linear scaling for reference."""
    ours = [d for d in runs if "unavailable" not in d and d.get("impl", "ours") == "ours"]
    if not ours:
        return []
    series = collections.defaultdict(list)
    for d in ours:
        series[d.get("config", {}).get("workload", "?")].append((d["n_gpus"], d["value"]))
        for dt in ("f16", "fp8"):
            r = (d.get("sharded") or {}).get(dt)
            if r:
                series[f"sharded {dt} GEMM"].append((d["n_gpus"], r["gemm_tflops_all_gpus"]))
                fu = r.get("fused_gather") or {}
                if "tflops_all_gpus" in fu:
                    series[f"sharded {dt} GEMM + gather"].append((d["n_gpus"], fu["tflops_all_gpus"]))
    gpus = sorted({n for pts in series.values() for n, _ in pts})
    ys = [v for pts in series.values() for _, v in pts]
    c = Svg("Whole-box TFLOP/s vs GPU count", "GPUs", "TFLOP/s (all GPUs)", gpus, ys, xlog=2 if len(gpus) > 1 else 0)
    c.xticks(gpus)
    for i, (name, pts) in enumerate(sorted(series.items())):
        c.line(pts, PALETTE[i % len(PALETTE)], name)
    os.makedirs(outdir, exist_ok=True)
    with open(os.path.join(outdir, "scaling.svg"), "w") as f:
        f.write(c.text())
    return ["![TFLOP/s vs GPU count](scaling.svg)", ""]


def render(csv_rows: list[dict], runs: list[dict], charts: str | None = None) -> str:
    out = ["# GEMM report", ""]
    if csv_rows:
        out += ["## gemm_bench rows", ""]
        if charts:
            out += device_charts(csv_rows, charts)
        out += size_tables(csv_rows)
    if runs:
        out += ["## bench.py runs by GPU count", ""]
        if charts:
            out += scaling_chart(runs, charts)
        out += scaling_table(runs)
    return "\n".join(out) + "\n"


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("csv", nargs="?", help="gemm_bench output (bench.csv schema)")
    ap.add_argument("--bench-json", action="append", default=[], help="file of bench.py JSON lines (repeatable)")
    ap.add_argument("--out", help="write here instead of stdout")
    ap.add_argument("--charts", help="directory for the SVG charts (linked from the report)")
    a = ap.parse_args(argv)
    rows = load_csv(a.csv) if a.csv else []
    runs = [d for p in a.bench_json for d in load_json_lines(p)]
    text = render(rows, runs, a.charts)
    if a.out:
        with open(a.out, "w") as f:
            f.write(text)
    else:
        print(text, end="")


if __name__ == "__main__":
    main()
