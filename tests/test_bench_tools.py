"""Host-side tooling of bench.py (no GPU): the ncu launch-list summary that
the committed step profiles are made with."""
import bench

_HDR = ('"ID","Process ID","Process Name","Host Name","Kernel Name","Context","Stream","Block Size",'
        '"Grid Size","Device","CC","Section Name","Metric Name","Metric Unit","Metric Value"')


def _row(i, name, ns, metric="gpu__time_duration.sum"):
    return (f'"{i}","1","python3","127.0.0.1","{name}","1","13","(256, 1, 1)","(72, 1, 1)","0","10.0",'
            f'"Command line profiler metrics","{metric}","ns","{ns}"')


def test_summarize_ncu_groups_kernels_by_readable_name(tmp_path, capsys):
    lines = ["==PROF== Connected to process 1", "==PROF== Disconnected from process 1", _HDR,
             _row(0, "void unnamed>::gemv_kernel<4, 1, 1, 2>(QTile, ActIn, int, Epi, StepIO, float *)", "5,000"),
             _row(1, "void unnamed>::gemv_kernel<4, 1, 1, 2>(QTile, ActIn, int, Epi, StepIO, float *)", "3000"),
             _row(2, "void unnamed>::tc_gemv_kernel<8, 3>(QTile, ActIn, int, Epi, StepIO, float *)", "4000"),
             _row(3, "void unnamed>::tc_gemm_kernel<4, 2>(CUtensorMap_st, QTile, int, __half *, int, int, "
                     "StepIO, float *)", "6000"),
             _row(4, "unnamed>::attn_pv_kernel(AttnArgs, int)", "2000"),
             _row(5, "unnamed>::attn_pv_kernel(AttnArgs, int)", "99", metric="dram__bytes_read.sum")]
    path = tmp_path / "launches.csv"
    path.write_text("\n".join(lines) + "\n")
    assert bench.summarize_ncu(str(path)) == 0
    out = capsys.readouterr().out.splitlines()
    table = {ln[:48].strip(): ln[48:].split() for ln in out[1:]}
    assert table["gemv_kernel<int4, nt8=1, resid>"] == ["2", "8.0", "40.0%"]
    assert table["tc_gemv_kernel<int8, swiglu>"] == ["1", "4.0", "20.0%"]
    assert table["tc_gemm_kernel<int4, 2 issuers>"] == ["1", "6.0", "30.0%"]
    assert table["attn_pv_kernel"] == ["1", "2.0", "10.0%"]   # the dram row is not a duration
    assert table["total"] == ["5", "20.0"]
    # largest total first
    assert out[1].startswith("gemv_kernel<int4, nt8=1, resid>")
