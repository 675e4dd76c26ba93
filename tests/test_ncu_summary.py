"""The ncu raw-page summariser on a synthetic capture (no GPU, no ncu run)."""
from nexar_b200.bench.ncu_summary import load_peaks, parse_raw_csv, summarise

RAW = '''"ID","Process ID","Process Name","Host Name","Kernel Name","Context","Stream","dram__bytes_read.sum","dram__bytes_write.sum","gpu__time_duration.sum","launch__registers_per_thread","sm__pipe_tensor_cycles_active.avg.pct_of_peak_sustained_active","sm__warps_active.avg.pct_of_peak_sustained_active"
"","","","","","","","Mbyte","Mbyte","usecond","register/thread","%","%"
"0","123","python","box","k_gemm_bf16_2sm","1","7","169.20","51.00","175.60","206","90.10","12.50"
"1","123","python","box","k_ln_bwd","1","7","37.80","0.02","23.90","254","0.00","40.00"
'''


def test_parse_and_summarise():
    recs = parse_raw_csv(RAW)
    assert [r["kernel"] for r in recs] == ["k_gemm_bf16_2sm", "k_ln_bwd"]
    g = recs[0]
    assert abs(g["duration"] - 175.6e-6) < 1e-12
    assert abs(g["dram_read"] - 169.2e6) < 1 and abs(g["dram_write"] - 51e6) < 1
    assert g["regs"] == 206 and g["tensor_active"] == 90.1
    peaks = {"hbm_gbs": 6543.4, "bf16_tflops": 1660.7, "source": "measured"}
    flops = 2 * 8192 * 4096 * 4096
    table = summarise(recs[:1], peaks, flops=flops)
    assert "k_gemm_bf16_2sm" in table and "of measured peak" in table
    tf = flops / 175.6e-6 / 1e12
    assert f"{tf:.1f}" in table and f"({tf / 1660.7:.2f})" in table


def test_fallback_peaks_when_file_missing(tmp_path):
    p = load_peaks(str(tmp_path / "absent.json"))
    assert p["source"] == "fallback" and p["hbm_gbs"] == 6650.0
