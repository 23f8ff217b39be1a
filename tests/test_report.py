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
