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


def _man(hidden, inter, heads, kv_heads, hd, vocab, attn_bits, mlp_bits):
    q = lambda out, k, bits: {"bits": bits, "block": 64, "out": out, "in": k, "in_real": k}  # noqa: E731
    layer = {"q": q(heads * hd, hidden, attn_bits), "k": q(kv_heads * hd, hidden, attn_bits),
             "v": q(kv_heads * hd, hidden, attn_bits), "o": q(hidden, heads * hd, attn_bits),
             "gate": q(inter, hidden, mlp_bits), "up": q(inter, hidden, mlp_bits),
             "down": q(hidden, inter, mlp_bits)}
    return {"config": {"hidden": hidden, "intermediate": inter, "heads": heads, "kv_heads": kv_heads,
                       "head_dim": hd, "vocab": vocab},
            "quant": {"layers": {"0": layer}}, "embed_quant": {"bits": 8, "block": hidden}}


def test_step_profile_groups_bytes_and_shares():
    tman = _man(1536, 8960, 12, 2, 128, 151936, 4, 8)
    dman = _man(896, 4864, 14, 2, 64, 151936, 4, 4)
    prof = [("spec", "spec_prep", 1, 1.0), ("draft", "embed", 1, 1.0), ("draft", "down", 1, 6.0),
            ("draft", "attn_scores", 1, 2.0), ("spec", "spec_prep", 1, 1.0), ("draft", "embed", 1, 1.0),
            ("draft", "down", 1, 6.0), ("draft", "attn_scores", 1, 2.0), ("target", "gate_up", 5, 10.0)]
    g = {x["key"]: x for x in bench.step_profile_groups(prof, tman, dman, 600, 4)}
    assert g["draft.down"]["launches"] == 2 and g["draft.down"]["us"] == 12.0
    # int4 896x4864: codes + scales + 1 input row + 1 output row
    down = 896 * 4864 // 2 + 896 * (4864 // 64) * 2 + 4864 * 2 + 896 * 2
    assert g["draft.down"]["bytes_per_launch"] == down
    assert abs(g["draft.down"]["gbs"] - 2 * down / 12e3) < 0.1
    # attention of draft forward i reads the K rows of positions 0..600+i
    assert g["draft.attn_scores"]["bytes"] == 2 * 64 * 2 * (601 + 602)
    gu = 2 * (8960 * 1536 + 8960 * 24 * 2) + 5 * 1536 * 2 + 5 * 17920 * 2
    assert g["target.gate_up"]["bytes_per_launch"] == gu
    assert abs(sum(x["share"] for x in g.values()) - 1.0) < 1e-3
    assert bench.step_profile_groups(prof, tman, dman, 600, 4)[0]["key"] == "draft.down"
