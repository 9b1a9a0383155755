"""Generated plasma code compiles with NVRTC for sm_100a in both storage
modes (no GPU needed), structurally equal groups share kernels, and the
backward write plan overwrites each gradient slot exactly once per step."""
import ctypes

import pytest

from nvrtc_check import compile_source
from oracle.tkm_abi import bind, compile_graph
from test_graph_cpu import DSL


def lib():
    from tokamak_b200 import engine
    return bind(engine())


def source_of(dsl, batch):
    L = lib()
    g = compile_graph(L, dsl, batch)
    p = L.tkm_codegen_cuda_string(ctypes.byref(g))
    assert p
    return ctypes.string_at(p).decode(), g


@pytest.mark.parametrize("name", ["llama_c1", "gqa_qknorm_rope_scaled", "twin_custom", "image_like", "rules",
                                  "residual_of_input"])
@pytest.mark.parametrize("act_bytes", [2, 4])
def test_generated_code_compiles_for_sm100a(name, act_bytes):
    src, _ = source_of(DSL[name], 4)
    assert src.startswith("// tokamak-b200 plasma codegen v1")
    ok, log, size = compile_source(src, act_bytes)
    assert ok, log[:4000]
    assert size > 0


def test_identical_layers_share_kernels():
    src, g = source_of(DSL["llama_c1"], 4)
    assert g.num_groups == 13
    assert "in 6 kernel classes" in src
    assert src.count("extern \"C\" __global__") < 3 * 6 + 1


def test_unsupported_groups_are_reported():
    src, _ = source_of("input: 8x8x4\nflow:\n  a: RandFlipX -> RandNoise -> FC(10) -> SoftmaxCE\n", 2)
    assert "#error" in src and "augmentation" in src


def test_residual_of_group_input_sums_before_one_store():
    """A residual whose skip is the group's own input: the Add branch
    gradient and d(input) share one slot, so the backward sums them in
    registers and stores once (no second write through an aliasing pointer)."""
    src, _ = source_of(DSL["residual_of_input"], 4)
    bwd = src[src.index("TKM_KNAME(bwd)"):]
    assert "tdbr" in bwd
    assert "tkm_st<TKG_VP>(a" in bwd or "tkm_st_add<TKG_VP>(a" in bwd


class RowGeom(ctypes.Structure):
    """TkmRowGeom (tokamak_b200/host/tkm_internal.h)."""
    _fields_ = [(n, ctypes.c_int) for n in ("C", "C2", "vp", "nch", "tpr", "kch", "rpb", "threads", "ncb", "rows",
                                              "fwd_grid", "persist")]


def test_row_geometry_of_configuration_3_groups():
    """The geometry the generator gives configuration 3's groups in bf16: a
    normalisation group keeps whole 4096-wide rows on 256 threads (two 16-byte
    chunks each), the SwiGLU twin epilogue splits an 11008-wide row over two
    column blocks of up to 1024 threads, a one-input Bias over 32000-wide rows
    over column blocks of at most 256 threads, and the backward uses the
    forward's geometry."""
    from tokamak_b200 import engine
    L = lib()
    E = engine()
    E.tkm_row_geom.restype = None
    E.tkm_row_geom_bwd.restype = None
    chain = ("input: 1x64x4096\nflow:\n  r: {\n    branch: FC(4096)\n    skip: Identity\n  } -> Add\n"
             "  f: RMSNorm -> {\n    gate: FC(11008) -> SiLU\n    up: FC(11008)\n  } -> Mul -> FC(10) -> SoftmaxCE\n")
    ce = "input: 1x32x512\nflow:\n  h: FC(32000) -> SoftmaxCE\n"
    seen = {}
    for dsl in (chain, ce):
        g = compile_graph(L, dsl, 1)
        for i in range(g.num_groups):
            grp = g.groups[i]
            fwd, bwd = RowGeom(), RowGeom()
            E.tkm_row_geom(ctypes.byref(g), ctypes.byref(grp), 2, ctypes.byref(fwd))
            E.tkm_row_geom_bwd(ctypes.byref(g), ctypes.byref(grp), 2, ctypes.byref(bwd))
            assert bytes(fwd) == bytes(bwd)
            kind = "twin" if grp.is_twin_epilogue else ("norm" if grp.has_norm else "elem")
            seen[(kind, grp.C)] = (fwd.vp, fwd.nch, fwd.kch, fwd.tpr, fwd.ncb, fwd.threads)
    assert seen[("norm", 4096)] == (4, 512, 2, 256, 1, 256)
    assert seen[("twin", 11008)] == (4, 1376, 1, 704, 2, 704)
    assert seen[("elem", 32000)] == (4, 4000, 1, 256, 16, 256)
