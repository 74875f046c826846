"""CPU tests of the C ABI library: it loads, exports every function include/b2g_gemm.h
declares, validates options, and its persistent tile order is a bijection for every grid
shape (including the ones where the reference's strip remap, mmm.cpp:1219-1236, is not).
No compute call is made here (no GPU)."""
import ctypes

import pytest


def test_library_exports_every_declared_symbol(b2g):
    L = b2g.load()
    names = b2g.declared_symbols()
    assert len(names) >= 10
    missing = [n for n in names if not hasattr(L, n)]
    assert not missing, missing


def test_version_and_error_string(b2g):
    assert "sm_100a" in b2g.version()
    assert isinstance(b2g.load().b2g_last_error_string(), bytes)


def test_options_roundtrip_and_validation(b2g):
    for key, val in [("cta_group", 2), ("raster_group", 4), ("timeout_ns", 123456789),
                     ("force_generic", 1), ("fault_flags", 0), ("tile_n", 512), ("tile_n", 128),
                     ("store_hint", 1), ("split_k", 3), ("tail_split", 0), ("serial_fixup", 1),
                     ("pdl", 0), ("cluster_fixup", 0)]:
        old = b2g.get_option(key)
        b2g.set_option(key, val)
        assert b2g.get_option(key) == val
        b2g.set_option(key, old)
    with pytest.raises(b2g.B2GError):
        b2g.set_option("no_such_option", 1)
    with pytest.raises(b2g.B2GError):
        b2g.set_option("cta_group", 3)
    with pytest.raises(b2g.B2GError):
        b2g.set_option("tile_n", 384)
    assert b2g.get_option("no_such_option") == -1


def test_invalid_arguments_rejected_without_gpu(b2g):
    """Argument validation runs before any CUDA call."""
    L = b2g.load()
    # negative dims
    assert L.b2g_gemm_f16_f32(None, None, None, -1, 4, 4, 4, 4, 4, None) == b2g.ERR_INVALID_ARG
    # lda < K
    assert L.b2g_gemm_f16_f32(None, None, None, 4, 4, 8, 4, 4, 4, None) == b2g.ERR_INVALID_ARG
    assert b"leading dimension" in L.b2g_last_error_string()
    # mismatched contraction modes
    a = (ctypes.c_int64 * 5)(1, 1, 4, 2, 8)
    b = (ctypes.c_int64 * 3)(2, 4, 8)
    c = (ctypes.c_int64 * 4)(1, 1, 4, 8)
    st5 = (ctypes.c_int64 * 5)(0, 0, 16, 8, 1)
    st3 = (ctypes.c_int64 * 3)(32, 8, 1)
    st4 = (ctypes.c_int64 * 4)(0, 0, 8, 1)
    rc = L.b2g_contract5d_f16_f32(None, a, st5, None, b, st3, None, c, st4, None)
    assert rc == b2g.ERR_INVALID_ARG
    assert b"contracted modes" in L.b2g_last_error_string()
    # null shape array
    rc = L.b2g_contract5d_f16_f32(None, None, st5, None, b, st3, None, c, st4, None)
    assert rc == b2g.ERR_INVALID_ARG
    # empty problem: nothing to do, no device needed
    assert L.b2g_gemm_f16_f32(None, None, None, 0, 4, 4, 4, 4, 4, None) == b2g.OK
    assert b2g.last_path() == b2g.PATH_EMPTY
    assert L.b2g_gemm_f16_f32_noalloc(None, None, None, 4, 0, 4, 4, 4, 4, None) == b2g.OK
    assert b2g.last_path() == b2g.PATH_EMPTY
    assert L.b2g_gemm_batched(None, None, None, 0, 4, 4, 4, 4, 4, 4, 16, 16, 16, None) == b2g.OK
    # epilogue, operand-type and batch arguments
    assert L.b2g_gemm_epilogue(None, None, None, 4, 4, 4, 4, 4, 4, 0, 1.0, 0.0, None, 7,
                               None) == b2g.ERR_INVALID_ARG
    assert b"output type" in L.b2g_last_error_string()
    assert L.b2g_gemm_epilogue(None, None, None, 4, 4, 4, 4, 4, 4, 0, 1.0, 1.0, None,
                               b2g.DTYPE_F16, None) == b2g.ERR_INVALID_ARG
    assert b"beta = 0" in L.b2g_last_error_string()
    assert L.b2g_gemm_typed(None, None, None, 4, 4, 4, 4, 4, 4, 9, 1.0, 0.0,
                            None) == b2g.ERR_INVALID_ARG
    assert L.b2g_gemm_batched(None, None, None, -1, 4, 4, 4, 4, 4, 4, 16, 16, 16,
                              None) == b2g.ERR_INVALID_ARG
    # the slot sum: count, self and slot alignment are checked first; an empty C needs nothing
    assert L.b2g_gemm_sum_slots(None, None, None, 4, 4, 4, 4, 4, 4, None, 16, 0, 0, None, 0,
                                None) == b2g.ERR_INVALID_ARG
    assert L.b2g_gemm_sum_slots(None, None, None, 4, 4, 4, 4, 4, 4, None, 16, 2, 2, None, 0,
                                None) == b2g.ERR_INVALID_ARG
    assert L.b2g_gemm_sum_slots(None, None, None, 4, 4, 4, 4, 4, 4, None, 16, 2, 0, None, 0,
                                None) == b2g.ERR_INVALID_ARG
    assert L.b2g_gemm_sum_slots(None, None, None, 4, 4, 4, 4, 4, 4, 4096 + 4, 16, 2, 0, None,
                                0, None) == b2g.ERR_INVALID_ARG
    assert b"16-byte aligned" in L.b2g_last_error_string()
    assert L.b2g_gemm_sum_slots(None, None, None, 4, 4, 4, 4, 4, 4, 4096, 12, 2, 0, None, 0,
                                None) == b2g.ERR_INVALID_ARG
    assert L.b2g_gemm_sum_slots(None, None, None, 0, 4, 4, 4, 4, 4, 4096, 16, 2, 0, None, 0,
                                None) == b2g.OK
    # multi-GPU plans: null plan / communicator rejected, destroying a null plan is a no-op
    assert L.b2g_gemm_sharded_k_p2p(None, None, None, None, 4, 4, 4, 4, 4, 4,
                                    None) == b2g.ERR_INVALID_ARG
    plan = ctypes.c_void_p()
    assert L.b2g_rs_plan_create(None, 4, 4, ctypes.byref(plan)) == b2g.ERR_INVALID_ARG
    assert L.b2g_rs_plan_destroy(None) == b2g.OK
    assert L.b2g_chain_plan_destroy(None) == b2g.OK


@pytest.mark.parametrize("num_m,num_n,group", [
    (1, 1, 8), (64, 32, 8), (64, 32, 16), (32, 32, 8), (40, 8, 32), (48, 64, 32), (7, 13, 3),
    (13, 7, 4), (1, 257, 8), (257, 1, 8), (100, 3, 7), (33, 112, 8), (5, 5, 1), (9, 2, 100)])
def test_tile_order_is_bijection(b2g, num_m, num_n, group):
    seen = set()
    for t in range(num_m * num_n):
        tm, tn = b2g.tile_coord(t, num_m, num_n, group)
        assert 0 <= tm < num_m and 0 <= tn < num_n
        seen.add((tm, tn))
    assert len(seen) == num_m * num_n


def _reference_strip_remap(bx, by, gx, gy):
    """Restatement of the reference's block swizzle (mmm.cpp:1219-1236) for comparison."""
    sw = 32 if gx >= 32 else gx
    block_id = by * gx + bx
    per_group = sw * gy
    group_id, lane = block_id // per_group, block_id % per_group
    x = group_id * sw + lane % sw
    y = lane // sw
    if x >= gx:
        x, y = bx, by
    return x, y


def test_reference_strip_remap_is_not_a_bijection_where_ours_is(b2g):
    """On a 40 x 8 block grid the reference remap repeats tiles and leaves others unvisited;
    the library's order visits each tile once."""
    gx, gy = 40, 8
    ref = {_reference_strip_remap(x, y, gx, gy) for y in range(gy) for x in range(gx)}
    assert len(ref) < gx * gy
    ours = {b2g.tile_coord(t, gy, gx, 8) for t in range(gx * gy)}
    assert len(ours) == gx * gy


def test_cpp_header_compiles_links_and_validates(b2g, tmp_path):
    """The C++ drop-in surface (include/b2g_gemm.hpp) builds against libb2g_gemm.so; the
    program calls only entry points that need no GPU (argument validation, partition, tile
    order) and maps a failing status to b2g::Error."""
    import os
    import shutil
    import subprocess
    from conftest import ROOT
    cxx = shutil.which("g++")
    if not cxx:
        pytest.skip("no g++")
    src = tmp_path / "dropin.cpp"
    src.write_text(r'''
#include <cstdio>
#include "b2g_gemm.hpp"
int main() {
  // the reference's GEMM(A, B, C, M, N, K) with a bad size: a status code, not an exit
  int rc = b2g::GEMM(nullptr, nullptr, nullptr, -1, 8, 8);
  if (rc != B2G_ERR_INVALID_ARG) return 1;
  try { b2g::check(rc); return 2; } catch (const b2g::Error& e) { if (e.code() != rc) return 3; }
  if (b2g::GEMM(nullptr, nullptr, nullptr, 0, 8, 8) != B2G_OK) return 4;   // empty problem
  int64_t r0, n;
  if (b2g_slab_rows(32768, 8, 3, &r0, &n) != B2G_OK || r0 != 12288 || n != 4096) return 5;
  int tm, tn;
  b2g_tile_coord(5, 3, 4, 2, &tm, &tn);
  std::printf("%s %d %d\n", b2g_version(), tm, tn);
  return 0;
}
''')
    exe = tmp_path / "dropin"
    libdir = os.path.join(ROOT, "rdna4-gemm-wmma_b200")
    res = subprocess.run([cxx, "-std=c++17", str(src), "-I", os.path.join(ROOT, "include"),
                          "-L", libdir, "-lb2g_gemm", "-Wl,-rpath," + libdir, "-o", str(exe)],
                         capture_output=True, text=True)
    assert res.returncode == 0, res.stderr
    run = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert run.returncode == 0, (run.returncode, run.stdout, run.stderr)
    assert "sm_100a" in run.stdout


@pytest.mark.parametrize("shape,plan", [
    # (M, N, K) -> (CTAs per tile, tile width, K splits, unsplit tiles) on 148 SMs
    ((8192, 8192, 8192), (2, 512, 1, 512)),         # 256x512 pair tiles
    ((8192, 4096, 8192), (2, 512, 2, 222)),         # configs[2] GEMM view: tail wave split 2 ways
    ((8192, 28672, 8192), (2, 512, 4, 1776)),       # configs[3]: 16 tail tiles split 4 ways
    ((16384, 16384, 4096), (2, 512, 1, 2048)),      # configs[3]: whole waves
    ((128, 8192, 8192), (1, 256, 4, 0)),            # configs[3] skinny: 32 tiles x 4 splits
    ((1024, 1024, 1024), (1, 128, 2, 0)),           # configs[0]: 64 tiles x 2 splits of 8 blocks
    ((256, 8192, 8192), (1, 256, 2, 0)),
    ((128, 2048, 8192), (1, 128, 8, 0)),
    ((512, 512, 2048), (1, 128, 4, 0)),             # four splits of 8 K blocks
    ((256, 512, 1024), (1, 128, 2, 0)),
    ((4096, 512, 1024), (1, 128, 1, 128)),          # tie: no 8-block splits
    ((2048, 2048, 2048), (2, 256, 1, 64)),          # no split: 256x256 pairs, same CTAs
    ((1024, 4096, 4096), (2, 256, 1, 64)),
    ((2048, 4096, 4096), (2, 512, 1, 64)),          # one wave of 512-wide pair tiles
    ((3072, 3072, 3072), (2, 512, 1, 72)),
])
def test_plan_preview_choices(b2g, shape, plan):
    """The launch plan for the BASELINE shapes and the small and mid shapes whose choice was
    measured: split-K units of the width that fills the SMs best (ties to 128x256), else
    256x256 pair tiles when no width splits, and 512-wide pair tiles whenever their waves fill
    the pairs as well as 256-wide ones."""
    assert b2g.plan_preview(*shape) == plan


@pytest.mark.parametrize("shape", [(128, 8192, 8192), (256, 8192, 8192), (8192, 8192, 8192),
                                   (128, 2048, 8192), (1024, 1024, 1024)])
def test_plan_preview_half_height_pairs_only_when_forced(b2g, shape):
    """The planner never chooses half-height pair tiles (64 A rows per CTA); pair_rows=64
    forces them (CTA pairs, 256-wide tiles) unless the caller also forces one-CTA tiles."""
    from gpu_util import options
    assert b2g.plan_preview(*shape, rows=True)[4] == 128
    with options(b2g, pair_rows=64):
        cg, bn, _, _, rows = b2g.plan_preview(*shape, rows=True)
        assert (cg, bn, rows) == (2, 256, 64)
    with options(b2g, pair_rows=64, cta_group=1):
        assert b2g.plan_preview(*shape, rows=True)[4] == 128


def test_plan_preview_follows_options(b2g):
    from gpu_util import options
    with options(b2g, cta_group=1, tile_n=256, split_k=3):
        assert b2g.plan_preview(384, 1024, 2240) == (1, 256, 3, 0)
    with options(b2g, tail_split=0):
        assert b2g.plan_preview(8192, 4096, 8192) == (2, 512, 1, 256)
    with pytest.raises(b2g.B2GError):
        b2g.plan_preview(0, 8, 8)


def test_plan_preview_invariants(b2g):
    """Random shapes, operand types and SM counts: the launch plan is always one the kernel can
    run.  Legal tile shapes; one-CTA tiles split at most 8 ways (the largest cluster of the
    cluster fix-up), pairs at most 16; every split keeps at least 16 K blocks (8 when one-CTA
    tiles split every tile); the split units
    of one launch fit in the resident CTA groups; unsplit plans run every tile whole."""
    from hypothesis import given, settings, strategies as st

    @settings(max_examples=400, deadline=None)
    @given(M=st.integers(1, 40000), N=st.integers(1, 40000), K=st.integers(1, 70000),
           dtype=st.sampled_from([0, 1, 2, 3]), sms=st.sampled_from([148, 132, 74, 16, 2]))
    def check(M, N, K, dtype, sms):
        cg, bn, splits, full, rows = b2g.plan_preview(M, N, K, dtype, sms, rows=True)
        assert cg in (1, 2) and bn in (128, 256, 512) and rows in (64, 128)
        assert not (cg == 1 and bn == 512) and not (bn == 128 and cg == 2)
        assert rows == 128 or (cg == 2 and bn == 256)
        esz = 2 if dtype < 2 else 1
        k_iters = -(-K * esz // 128)  # a K block is 128 bytes of K
        tiles = -(-(-(-M // rows)) // cg) * -(-N // bn)
        # half-height pairs split only through the cluster fix-up: at most 4 splits, no tail
        assert 1 <= splits <= (4 if rows == 64 else 8 if cg == 1 else 16)
        assert rows == 128 or splits == 1 or full == 0
        assert splits <= max(1, k_iters)
        assert 0 <= full <= tiles
        if splits == 1:
            assert full == tiles
        else:
            assert -(-k_iters // splits) >= (8 if (cg == 1 and rows == 128 and full == 0) else 16)
            groups = sms if cg == 1 else max(1, sms // 2)
            assert (tiles - full) * splits <= groups

    check()
