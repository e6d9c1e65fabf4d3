"""Generate the golden vectors in ``tests/golden/golden.pt`` from the reference's own code.

Run where the reference checkout exists (it is not needed afterwards; the tests only read the
fixture file):

    REF=/path/to/reference python tests/golden/make_golden.py

What is produced, and by which reference code:
  relayout_*   ``to_word_ncontig`` of gemv/moe_gemv_int2_tab.py:100-109 on seeded bytes
  tab_*        the Triton word-layout GEMV ``moe_gemv_int2_tab`` (gemv/moe_gemv_int2_tab.py:23-85)
               executed by the Triton CPU interpreter on CPU tensors with hand-built address tables:
               the w13 form (shared activation, TOP_K=3, N=200 not a block multiple) and the w2 form
               (per-row activations, TOP_K=1, routed weights), f16 and bf16 scales
  byte_*       the byte-layout GEMV ``gemv_int2`` (gemv/moe_gemv_int2.py:23-83) under the interpreter
  zp_*         ``make_int2_experts(has_zp=True)`` and ``torch_moe`` of the reference's synthetic unit
               test (series-0002 patch, test_moe_wna16_int2.py:1936-1973), taken from the patch text
               and executed as-is
  int8_*       ``pack_int8_gptq`` / ``unpack_int8_gptq`` of scripts/requant_int8.py:32-63
"""
from __future__ import annotations

import os
import sys

os.environ["TRITON_INTERPRET"] = "1"          # must precede the triton import
REF = os.environ.get("REF")
if not REF:
    raise SystemExit("set REF to the reference checkout (see the module docstring)")
OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden.pt")
SERIES = os.path.join(REF, "sglang/upstream/series-base/0002-feat-moe_wna16-2-bit-experts-expert-streaming-N-cont.patch")

import torch                                   # noqa: E402
import torch.nn.functional as F                # noqa: E402

sys.path.insert(0, os.path.join(REF, "gemv"))
sys.path.insert(0, os.path.join(REF, "scripts"))
import moe_gemv_int2_tab as tabmod             # noqa: E402
import moe_gemv_int2 as bytemod                # noqa: E402
import requant_int8 as i8mod                   # noqa: E402


def cpu_tables(t: torch.Tensor) -> torch.Tensor:
    """int64 [E] base addresses of a CPU tensor's expert slices (what make_tables builds on a GPU)."""
    return torch.tensor([t.data_ptr() + e * t.stride(0) * t.element_size() for e in range(t.shape[0])],
                        dtype=torch.int64)


def series_test_helpers() -> dict:
    """Execute the helper functions of the reference unit test test_moe_wna16_int2.py, read from the
    series patch (the file is added by that patch; its lines start with '+')."""
    txt = open(SERIES, encoding="utf-8").read().splitlines()
    start = next(i for i, l in enumerate(txt) if l.startswith("+++ b/test/registered/unit/layers/quantization/test_moe_wna16_int2.py"))
    body = []
    for l in txt[start + 2:]:
        if l.startswith("diff --git") or l.startswith("-- "):
            break
        if l.startswith("+"):
            body.append(l[1:])
    src = "\n".join(body)
    a = src.index("def pack_2bit_along_last")
    b = src.index("class TestWordLayoutCPU")
    ns = {"torch": torch, "F": F}
    exec(compile(src[a:b], "test_moe_wna16_int2.py(helpers)", "exec"), ns)
    return ns


def main():
    out = {}
    g = torch.Generator().manual_seed(7)

    # ---- relayout
    u8 = torch.randint(0, 256, (2, 64, 64), dtype=torch.uint8, generator=g)
    out["relayout_in"] = u8
    out["relayout_out"] = tabmod.to_word_ncontig(u8)

    # ---- Triton word GEMV (interpreter)
    for sname, sdt in (("f16", torch.float16), ("bf16", torch.bfloat16)):
        E, K13, N13, K2, N2, topk = 6, 256, 200, 128, 256, 3
        w13 = torch.randint(-(2 ** 31), 2 ** 31, (E, K13 // 16, N13), dtype=torch.int32, generator=g)
        s13 = (torch.rand(E, K13 // 128, N13, generator=g) * 0.1 + 0.01).to(sdt)
        w2 = torch.randint(-(2 ** 31), 2 ** 31, (E, K2 // 16, N2), dtype=torch.int32, generator=g)
        s2 = (torch.rand(E, K2 // 128, N2, generator=g) * 0.1 + 0.01).to(sdt)
        ids = torch.randperm(E, generator=g)[:topk].to(torch.int32)
        x13 = torch.randn(1, K13, generator=g).to(torch.bfloat16)
        x2 = torch.randn(topk, K2, generator=g).to(torch.bfloat16)
        rw = (torch.rand(topk, generator=g) + 0.5).float()
        o13 = tabmod.moe_gemv_int2_tab(x13, cpu_tables(w13), cpu_tables(s13), ids, rw, N13, K13, w13.stride(1),
                                       s13.stride(1), top_k=topk, mul_routed_weight=False,
                                       scale_bf16=sdt == torch.bfloat16)
        o2 = tabmod.moe_gemv_int2_tab(x2, cpu_tables(w2), cpu_tables(s2), ids, rw, N2, K2, w2.stride(1),
                                      s2.stride(1), top_k=1, mul_routed_weight=True,
                                      scale_bf16=sdt == torch.bfloat16)
        out.update({f"tab_{sname}_w13": w13, f"tab_{sname}_s13": s13, f"tab_{sname}_w2": w2,
                    f"tab_{sname}_s2": s2, f"tab_{sname}_ids": ids, f"tab_{sname}_x13": x13,
                    f"tab_{sname}_x2": x2, f"tab_{sname}_rw": rw, f"tab_{sname}_o13": o13.clone(),
                    f"tab_{sname}_o2": o2.clone()})

    # ---- byte-layout GEMV (interpreter)
    E, N, K, T = 4, 64, 512, 3
    qb = torch.randint(0, 256, (E, N, K // 4), dtype=torch.uint8, generator=g)
    sb = (torch.rand(E, N, K // 128, generator=g) * 0.05 + 0.01).to(torch.float16)
    eids = torch.tensor([2, 0, 3], dtype=torch.int32)
    xb = torch.randn(K, generator=g).to(torch.bfloat16)
    wt = torch.tensor([qb.data_ptr() + e * qb.stride(0) for e in range(E)], dtype=torch.int64)
    st = torch.tensor([sb.data_ptr() + e * sb.stride(0) * 2 for e in range(E)], dtype=torch.int64)
    ob = bytemod.gemv_int2(xb, wt, st, eids, N, K)
    out.update({"byte_q": qb, "byte_s": sb, "byte_ids": eids, "byte_x": xb, "byte_out": ob.clone()})

    # ---- per-group zero points: the reference unit test's own synthetic experts and torch MoE
    ns = series_test_helpers()
    gz = torch.Generator().manual_seed(1234)
    e, n, k, grp, topk, m = 4, 128, 128, 128, 2, 3
    w1_ref, w1_q, w1_s, w1_zp = ns["make_int2_experts"](e, 2 * n, k, grp, True, torch.bfloat16, gz)
    w2_ref, w2_q, w2_s, w2_zp = ns["make_int2_experts"](e, k, n, grp, True, torch.bfloat16, gz)
    a = (torch.randn((m, k), generator=gz) / 10).to(torch.bfloat16)
    score = torch.randn((m, e), generator=gz).to(torch.bfloat16)
    moe = ns["torch_moe"](a, w1_ref, w2_ref, score, topk)
    out.update({"zp_w1_ref": w1_ref, "zp_w1_q": w1_q, "zp_w1_s": w1_s, "zp_w1_zp": w1_zp,
                "zp_w2_ref": w2_ref, "zp_w2_q": w2_q, "zp_w2_s": w2_s, "zp_w2_zp": w2_zp,
                "zp_a": a, "zp_score": score, "zp_topk": torch.tensor(topk), "zp_moe": moe})
    qv = torch.randint(0, 4, (2, 8, 64), generator=torch.Generator().manual_seed(5))
    out["zp_words_vals"] = qv
    out["zp_words"] = ns["pack_words_along_k"](qv)
    out["zp_bytes"] = ns["pack_2bit_along_last"](qv)

    # ---- INT8 packing of the dense projections
    wd = (torch.randn(64, 256, generator=g) * 0.05).to(torch.bfloat16)
    qw, qz, sc = i8mod.pack_int8_gptq(wd)
    out.update({"int8_w": wd, "int8_qw": qw, "int8_qz": qz, "int8_sc": sc,
                "int8_deq": i8mod.unpack_int8_gptq(qw, qz, sc)})

    torch.save(out, OUT)
    print(f"wrote {OUT}: {len(out)} tensors, {os.path.getsize(OUT)} bytes")


if __name__ == "__main__":
    main()
