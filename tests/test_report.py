"""CPU: the Markdown report over the reference's bench.csv schema and bench.py JSON lines."""
import json

import report


def test_report_tables(tmp_path):
    csvp = tmp_path / "bench.csv"
    csvp.write_text(
        "device,sm,M,N,K,kernel,ms,tflops,pct_of_cublas,max_abs_err,pct_of_peak,dtype\n"
        '"NVIDIA B200",100,8192,8192,8192,tc_f16,0.764,1439.80,0.0,0.0112,64.0,f16\n'
        '"NVIDIA B200",100,8192,8192,8192,cublas_tc,0.743,1479.10,0.0,0.0112,65.7,f16\n'
        '"NVIDIA B200",100,1024,1024,1024,tc_fp8_amax,0.009,243.85,0.0,0.487,5.4,e4m3\n')
    runs = tmp_path / "runs.jsonl"
    lines = [{"impl": "ours", "n_gpus": n, "value": 1350.0 * n * 0.98 ** (n > 1), "ms_per_step": 0.8,
              "config": {"workload": "f16_gemm_8192x8192x8192_per_gpu"}, "e2e": {"value": 180.0},
              "gather": {"ms": 7.4, "fused": {"ms_per_step": 5.8}} if n > 1 else None} for n in (1, 2, 8)]
    lines.append({"impl": "reference", "unavailable": "x"})
    runs.write_text("noise\n" + "\n".join(json.dumps(d) for d in lines) + "\n")
    out = tmp_path / "report.md"
    report.main([str(csvp), "--bench-json", str(runs), "--out", str(out)])
    text = out.read_text()
    assert "| tc_f16 | f16 | 1439.8 | 97.3% of cublas_tc |" in text
    assert "M = 1024, N = 1024, K = 1024" in text
    assert text.index("M = 1024") < text.index("M = 8192")  # smaller problems first
    assert "| 8 | 10584.0 | 7.84 |" in text and "| 5.8 |" in text
    assert "reference" not in text.split("bench.py runs")[1]


def test_report_reads_the_reference_csv_schema(tmp_path):
    csvp = tmp_path / "bench.csv"
    csvp.write_text("device,sm,M,N,K,kernel,ms,tflops,pct_of_cublas,max_abs_err\n"
                    '"NVIDIA RTX 5090",120,4096,4096,4096,mma_warptile,1.0,137.4,90.0,0.0077\n')
    text = report.render(report.load_csv(str(csvp)), [])
    assert "| mma_warptile | - | 137.4 | - | - | 0.0077 |" in text


def test_report_svg_charts(tmp_path):
    """The reference's chart set (throughput vs size, % of library, bars, precision Pareto) and
    the GPU-count chart, written as standalone SVG that parses as XML."""
    import xml.etree.ElementTree as ET

    rows = ["device,sm,M,N,K,kernel,ms,tflops,pct_of_cublas,max_abs_err,pct_of_peak,dtype"]
    for n, (f16, lib, fp8, mx) in {1024: (207.0, 180.0, 274.0, 300.0), 4096: (1200.0, 1150.0, 2300.0, 4000.0),
                                   8192: (1440.0, 1400.0, 2900.0, 5600.0)}.items():
        rows += [f'"NVIDIA B200",100,{n},{n},{n},tc_f16,1,{f16},0,0.0112,0,f16',
                 f'"NVIDIA B200",100,{n},{n},{n},cublas_tc,1,{lib},0,0.0112,0,f16',
                 f'"NVIDIA B200",100,{n},{n},{n},tc_fp8,1,{fp8},0,1.4,0,e4m3',
                 f'"NVIDIA B200",100,{n},{n},{n},tc_mxfp4,1,{mx},0,5.97,0,e2m1']
    csvp = tmp_path / "bench.csv"
    csvp.write_text("\n".join(rows) + "\n")
    runs = tmp_path / "runs.jsonl"
    sh = lambda n: {"f16": {"gemm_ms": 13.9 / n, "gemm_tflops_all_gpus": 1268.0 * n,  # noqa: E731
                            "fused_gather": {"ms_per_step": 5.75, "tflops_all_gpus": 3060.0} if n > 1 else {}}}
    runs.write_text("\n".join(json.dumps({"impl": "ours", "n_gpus": n, "value": 1400.0 * n, "ms_per_step": 0.8,
                                          "config": {"workload": "f16_gemm_8192x8192x8192_per_gpu"},
                                          "sharded": sh(n)}) for n in (1, 2, 4, 8)) + "\n")
    charts = tmp_path / "charts"
    out = tmp_path / "report.md"
    report.main([str(csvp), "--bench-json", str(runs), "--out", str(out), "--charts", str(charts)])
    names = sorted(p.name for p in charts.iterdir())
    assert names == ["bars_sm100.svg", "pareto_sm100.svg", "pct_library_sm100.svg", "scaling.svg", "tflops_sm100.svg"]
    for p in charts.iterdir():
        root = ET.fromstring(p.read_text())
        assert root.tag.endswith("svg")
    assert "polyline" in (charts / "tflops_sm100.svg").read_text()
    text = out.read_text()
    for n in names:
        assert f"]({n})" in text
    assert "sharded record (strong scaling)" in text and "| 8 | f16 |" in text
