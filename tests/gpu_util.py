"""Helpers shared by the GPU parity tests: seeded inputs (host oracle generator, copied to
the device), the oracle comparison, and option scoping.  torch is used only to hold device
memory; every product computation goes through the C ABI."""
import contextlib

import numpy as np


def to_dev(torch, arr):
    t = torch.from_numpy(np.ascontiguousarray(arr))
    return t.cuda()


def padded_f16(torch, orc, rows, cols, ld, seed, offset=0):
    """rows x cols fp16 matrix (row pitch ld) holding the oracle sequence for the logical
    rows x cols matrix; the pad columns hold a different sequence so a kernel that reads
    them is caught."""
    logical = orc.uniform_f16((rows, cols), seed, offset)
    full = orc.uniform_f16((rows, ld), seed + 1000003, offset)
    full[:, :cols] = logical
    return logical, to_dev(torch, full)


def assert_close(orc, got, ref, K, max_a=1.0, max_b=1.0, what=""):
    bad, ma, mr, first = orc.check(got, ref, K, max_a, max_b)
    assert bad == 0, "%s: %d elements out of tolerance (max abs %.3g, max rel %.3g, first %d: got %r ref %r)" % (
        what, bad, ma, mr, first, np.asarray(got).ravel()[first], np.asarray(ref).ravel()[first])
    return ma, mr


# kernel variants of the tensor-core path: (CTAs per tile, tile width)
VARIANTS = [(1, 128), (1, 256), (2, 256), (2, 512)]
VARIANT_IDS = ["cta1_n128", "cta1_n256", "cta2_n256", "cta2_n512"]
# ... plus the 256 x 512 pair tile with four epilogue warps instead of the default eight (tile
# width "512w4") and the half-height pair tile (128 x 256 over a CTA pair, 64 A rows per CTA;
# tile width "256h"), which options() below selects
VARIANTS_W8 = VARIANTS + [(2, "512w4")]
VARIANT_W8_IDS = VARIANT_IDS + ["cta2_n512_epi4"]
VARIANTS_H = VARIANTS_W8 + [(2, "256h")]
VARIANT_H_IDS = VARIANT_W8_IDS + ["cta2_n256_half"]


@contextlib.contextmanager
def options(b2g, **kw):
    if kw.get("tile_n") == "256h":
        kw["tile_n"] = 256
        kw["pair_rows"] = 64
    elif kw.get("tile_n") == "512w4":
        kw["tile_n"] = 512
        kw["epi_warps"] = 4
    old = {k: b2g.get_option(k) for k in kw}
    try:
        for k, v in kw.items():
            b2g.set_option(k, v)
        yield
    finally:
        for k, v in old.items():
            b2g.set_option(k, v)
