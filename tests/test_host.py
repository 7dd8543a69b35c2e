"""Host-side checks that need no GPU: the C-ABI library loads and exports the
header's symbols, contract violations fail with the reference's messages
before any device work, host quantisers are byte-identical to the oracle, the
synthetic generator is shard-consistent, and the top-1 combine keeps the
first maximum."""
import re
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent


def header_symbols():
    txt = (ROOT / "include" / "focr_cuda.h").read_text()
    return sorted(set(re.findall(r"\b(focr_[a-z0-9_]+)\s*\(", txt)))


def test_library_exports_every_header_symbol():
    from franken_ocr_b200 import _lib

    syms = header_symbols()
    assert len(syms) >= 17
    for s in syms:
        assert hasattr(_lib.lib, s), f"missing export {s}"
    assert sorted(_lib.EXPORTS) == syms


def test_tier_string():
    from franken_ocr_b200 import simd

    assert simd.tier_string() == "sm100a"


@pytest.mark.parametrize("alen,blen,olen,msg", [
    (2, 1, 1, "igemm_s8s8: a.len 2 != m*k 1"),
    (1, 3, 1, "igemm_s8s8: b.len 3 != n*k 1"),
    (1, 1, 5, "igemm_s8s8: out.len 5 != m*n 1"),
])
def test_igemm_length_contract(alen, blen, olen, msg):
    from franken_ocr_b200 import simd

    with pytest.raises(simd.FocrError) as ei:
        simd.igemm_s8s8(np.zeros(alen, np.int8), np.zeros(blen, np.int8), 1, 1, 1,
                        np.zeros(olen, np.int32))
    assert str(ei.value) == msg and ei.value.code == -1


def test_igemm_overflow_messages():
    from franken_ocr_b200 import simd

    with pytest.raises(simd.FocrError, match="igemm_s8s8: m\\*k overflow"):
        simd.igemm_s8s8(np.zeros(0, np.int8), np.zeros(0, np.int8), 2**64 - 1, 2, 0,
                        np.zeros(0, np.int32))
    with pytest.raises(simd.FocrError, match="igemm_u8s8: m\\*n overflow"):
        simd.igemm_u8s8(np.zeros(0, np.uint8), np.zeros(0, np.int8), 2**64 - 1, 0, 2,
                        np.zeros(0, np.int32))


@pytest.mark.parametrize("k,group,msg", [(15, 16, "k 15 must be even"),
                                         (32, 8, "group 8 must be 16 or 32"),
                                         (48, 32, "group 32 must divide k 48")])
def test_int4_contract(k, group, msg):
    from franken_ocr_b200 import simd

    with pytest.raises(simd.FocrError, match=msg):
        simd.igemm_s4s8_packed(np.zeros(k, np.int8), np.zeros(k // 2, np.uint8),
                               np.zeros(1, np.float32), group, 1, k, 1, np.zeros(1, np.float32))


def test_empty_shapes_are_noops():
    from franken_ocr_b200 import simd

    out = np.zeros(0, np.int32)
    simd.igemm_s8s8(np.zeros(0, np.int8), np.zeros(0, np.int8), 0, 5, 0, out)


def test_top1_combine_first_max():
    from franken_ocr_b200.lmhead import top1_combine

    vals = np.array([[1.0, np.nan, 2.0], [3.0, np.nan, 2.0], [3.0, 5.0, 1.0]], np.float32)
    idx = np.array([[4, -1, 7], [20, -1, 21], [40, 41, 42]], np.int32)
    assert top1_combine(vals, idx).tolist() == [20, 41, 7]
    assert top1_combine(np.full((2, 1), np.nan, np.float32), np.full((2, 1), -1, np.int32)).tolist() == [0]


def test_host_quantisers_match_oracle(oracle):
    from franken_ocr_b200.quant import pack_int4_f32, quantize_int8_f32, unpack_int4

    g = np.random.default_rng(7)
    w = (g.standard_normal((37, 96), dtype=np.float32) * np.float32(0.02)).astype(np.float32)
    w[3] = 0.0
    w[5, :4] = [0.5, -0.5, 1.5, 127.0]
    q, s = quantize_int8_f32(w)
    qo, so = oracle.quantize_int8_weights(w)
    assert np.array_equal(q, qo) and np.array_equal(s.view(np.uint32), so.view(np.uint32))
    for group in (16, 32):
        p, gs = pack_int4_f32(w, group)
        po, gso = oracle.pack_int4(w, group)
        assert np.array_equal(p, po) and np.array_equal(gs, gso)
        assert np.array_equal(unpack_int4(p, 96).ravel(), oracle.unpack_to_i8(p, 37, 96))


def test_synth_shards_consistent():
    from franken_ocr_b200 import synth

    full = synth.moe_layer(3, hidden=64, inter=32, n_experts=8, topk=2)
    part = synth.moe_layer(3, hidden=64, inter=32, n_experts=8, topk=2, expert_begin=4, expert_count=2)
    for k in ("gate_w", "up_s", "down_w"):
        assert np.array_equal(full.arrays[k][4:6], part.arrays[k])
    assert np.array_equal(full.router, part.router)
    q, s = synth.lm_head(1, 50, hidden=32, row_begin=0, block=20)
    q2, s2 = synth.lm_head(1, 15, hidden=32, row_begin=17, block=20)
    assert np.array_equal(q[17:32], q2) and np.array_equal(s[17:32], s2)


def test_zipf_routing_is_skewed_and_distinct():
    from franken_ocr_b200 import synth

    idx, w = synth.zipf_routing(5, 256)
    assert all(len(set(r)) == 6 for r in idx.tolist())
    counts = np.bincount(idx.ravel(), minlength=64)
    top = np.sort(counts)[::-1]
    assert top[0] > 4 * max(top[-8:].mean(), 1)   # heavy head, light tail
    assert np.allclose(w.sum(1), 1.0, atol=1e-5) and (np.diff(w, axis=1) <= 0).all()


def test_status_word_check_reports_injected_expiry():
    """A status word with the expired-wait bit (injected on the host) maps to
    FOCR_E_TIMEOUT with a message; 0 maps to success.  Pure host logic."""
    from franken_ocr_b200._lib import FOCR_E_TIMEOUT, FOCR_OK, lib

    assert lib.focr_status_check(0) == FOCR_OK
    assert lib.focr_status_check(4) == FOCR_E_TIMEOUT
    msg = lib.focr_last_error().decode()
    assert "bounded device-side wait expired" in msg and "0x4" in msg


def test_libm_expf_table_recomputed():
    """Entry i of the device exp's table = bits of the double nearest
    2^(i/32), minus i << 47 (recomputed here at 60 digits)."""
    import struct
    from decimal import Decimal, getcontext

    getcontext().prec = 60
    txt = (ROOT / "franken_ocr_b200" / "csrc" / "libm_expf.h").read_text()
    got = [int(v, 16) for v in re.findall(r"0x([0-9a-f]{16})ULL", txt)]
    ln2 = Decimal(2).ln()
    want = []
    for i in range(32):
        b = struct.unpack("<Q", struct.pack("<d", float((ln2 * i / 32).exp())))[0]
        want.append((b - (i << 47)) & (2**64 - 1))
    assert got == want


def test_libm_expf_matches_glibc_on_every_float(tmp_path):
    """The device exp (csrc/libm_expf.h, compiled for the host here) equals
    this host's libm expf -- the function the reference's f32::exp calls --
    on all 2^32 inputs."""
    import subprocess

    src = tmp_path / "t.cc"
    src.write_text(r'''
#include <cmath>
#include <cstdio>
#include <cstring>
#include "libm_expf.h"
int main() {
    long bad = 0;
    #pragma omp parallel for reduction(+:bad) schedule(dynamic, 1 << 16)
    for (long u = 0; u < (1L << 32); u++) {
        float x; unsigned b = (unsigned)u; std::memcpy(&x, &b, 4);
        float r = expf(x), m = libm_expf(x);
        if (r != r && m != m) continue;
        if (std::memcmp(&r, &m, 4)) bad++;
    }
    std::printf("%ld\n", bad);
    return 0;
}
''')
    exe = tmp_path / "t"
    subprocess.run(["g++", "-O2", "-ffp-contract=off", "-fopenmp", "-I",
                    str(ROOT / "franken_ocr_b200" / "csrc"), str(src), "-o", str(exe), "-lm"],
                   check=True)
    out = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout
    assert out.strip() == "0"


def test_nccl_unique_id_is_128_bytes_or_unsupported():
    """The communicator bootstrap loads NCCL at run time: either a 128-byte
    id comes back, or FOCR_E_UNSUPPORTED says why (no library)."""
    import ctypes as C

    from franken_ocr_b200._lib import FOCR_E_UNSUPPORTED, FOCR_OK, lib

    buf = C.create_string_buffer(128)
    rc = lib.focr_nccl_unique_id(buf)
    assert rc in (FOCR_OK, FOCR_E_UNSUPPORTED)
    if rc == FOCR_E_UNSUPPORTED:
        assert b"nccl" in lib.focr_last_error().lower()
