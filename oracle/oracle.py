"""ctypes wrapper of the CPU oracle (``oracle/_build/libfocr_oracle.so``).

TEST INFRASTRUCTURE ONLY: imported by tests/, ``__graft_entry__.smoke()`` and
the CPU-baseline legs of bench.py -- never by the product package.  The C
sources (focr_oracle.c, cpu_baseline.c) restate the reference's Rust with
file:line citations; ``make -C oracle`` builds the library.
"""
from __future__ import annotations

import ctypes as C
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "_build" / "libfocr_oracle.so"


def build() -> Path:
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB_PATH


if not LIB_PATH.exists():
    build()
lib = C.CDLL(str(LIB_PATH))
vp, sz = C.c_void_p, C.c_size_t


class MoeLayerC(C.Structure):
    _fields_ = [
        ("hidden", sz), ("inter", sz), ("n_experts", sz), ("topk", sz), ("shared_inter", sz),
        ("norm_topk_prob", C.c_int), ("routed_scaling_factor", C.c_float),
        ("router", vp), ("gate_w", vp), ("gate_s", vp), ("up_w", vp), ("up_s", vp),
        ("down_w", vp), ("down_s", vp),
        ("sh_gate_w", vp), ("sh_gate_s", vp), ("sh_up_w", vp), ("sh_up_s", vp),
        ("sh_down_w", vp), ("sh_down_s", vp),
        ("group", sz), ("gate_p", vp), ("gate_gs", vp), ("up_p", vp), ("up_gs", vp),
        ("down_p", vp), ("down_gs", vp),
    ]


lib.oracle_sign_extend_nibble.restype = C.c_int8
lib.oracle_sign_extend_nibble.argtypes = [C.c_uint8]
lib.oracle_quantize_row_i8.restype = C.c_float
lib.oracle_quantize_row_i8_te.restype = C.c_float
lib.oracle_silu.restype = C.c_float
lib.oracle_silu.argtypes = [C.c_float]
lib.oracle_argmax_row.restype = C.c_uint32
lib.oracle_cpu_tier.restype = C.c_char_p
for _f in ("oracle_igemm_s8s8", "oracle_igemm_u8s8", "oracle_cpu_igemm_s8s8"):
    getattr(lib, _f).argtypes = [vp, vp, sz, sz, sz, vp]
lib.oracle_cpu_igemm_s8s8_mt.argtypes = [vp, vp, sz, sz, sz, vp, C.c_int]
lib.oracle_unpack_to_i8.argtypes = [vp, sz, sz, vp]
lib.oracle_igemm_s4s8_packed.argtypes = [vp, vp, vp, sz, sz, sz, sz, vp]
lib.oracle_quantize_row_i8.argtypes = [vp, sz, vp]
lib.oracle_quantize_row_i8_te.argtypes = [vp, sz, vp]
lib.oracle_quantize_int8_weights.argtypes = [vp, sz, sz, vp, vp]
lib.oracle_pack_int4.argtypes = [vp, sz, sz, sz, vp, vp]
lib.oracle_gemv_i8_prequant.argtypes = [vp, C.c_float, vp, vp, sz, sz, vp]
lib.oracle_gemv_i8.argtypes = [vp, vp, vp, sz, sz, vp]
lib.oracle_expert_i8.argtypes = [vp, sz, sz, vp, vp, vp, vp, vp, vp, vp]
lib.oracle_router_logits.argtypes = [vp, sz, vp, sz, vp]
lib.oracle_route.argtypes = [vp, sz, sz, vp, sz, sz, C.c_int, C.c_float, vp, vp]
lib.oracle_moe_decode.argtypes = [C.POINTER(MoeLayerC), vp, sz, vp, vp, vp]
lib.oracle_moe_decode_routed.argtypes = [C.POINTER(MoeLayerC), vp, sz, vp, vp, vp]
lib.oracle_moe_prefill.argtypes = lib.oracle_moe_decode.argtypes
lib.oracle_moe_prefill.restype = C.c_int
lib.oracle_moe_prefill_routed.argtypes = lib.oracle_moe_decode_routed.argtypes
lib.oracle_moe_prefill_routed.restype = C.c_int
lib.oracle_cpu_moe_decode.argtypes = [C.POINTER(MoeLayerC), vp, sz, vp, vp, vp, C.c_int]
lib.oracle_vocab_tile_ranges.argtypes = [sz, sz, vp, vp]
lib.oracle_rms_norm.argtypes = [vp, sz, sz, vp, C.c_float, vp]
lib.oracle_rope_table.argtypes = [vp, sz, sz, C.c_float, vp, vp]
lib.oracle_apply_rope.argtypes = [vp, sz, sz, sz, vp, vp]
lib.oracle_attention_decode.argtypes = [vp, vp, vp, sz, sz, vp, vp, sz, sz, sz, sz, vp]
lib.oracle_attention_decode.restype = C.c_int
lib.oracle_argmax_row.argtypes = [vp, sz]
lib.oracle_linear_i8.argtypes = [vp, sz, sz, vp, vp, sz, C.c_int, vp]
lib.oracle_swiglu_mlp_i8.argtypes = [vp, sz, sz, sz, vp, vp, vp, vp, vp, vp, C.c_int, vp]
lib.oracle_attention_prefill.argtypes = [vp, vp, vp, sz, sz, sz, vp]
lib.oracle_attention_prefill.restype = C.c_int
lib.oracle_silu_mul.argtypes = [vp, vp, sz, vp]
lib.oracle_cpu_linear_i8.argtypes = [vp, sz, sz, vp, vp, sz, C.c_int, vp, C.c_int]


def _p(a):
    return None if a is None else a.ctypes.data


def _c(a, dt):
    return np.ascontiguousarray(a, dtype=dt)


def igemm_s8s8(a, b, m, k, n, out):
    lib.oracle_igemm_s8s8(_p(a), _p(b), m, k, n, _p(out))


def igemm_u8s8(a, b, m, k, n, out):
    lib.oracle_igemm_u8s8(_p(a), _p(b), m, k, n, _p(out))


def cpu_igemm_s8s8(a, b, m, k, n, out, threads=1):
    if threads == 1:
        lib.oracle_cpu_igemm_s8s8(_p(a), _p(b), m, k, n, _p(out))
    else:
        lib.oracle_cpu_igemm_s8s8_mt(_p(a), _p(b), m, k, n, _p(out), threads)


def cpu_tier() -> str:
    return lib.oracle_cpu_tier().decode()


def sign_extend_nibble(n: int) -> int:
    return int(lib.oracle_sign_extend_nibble(n))


def unpack_to_i8(packed, n, k):
    out = np.empty(n * k, np.int8)
    lib.oracle_unpack_to_i8(_p(_c(packed, np.uint8)), n, k, _p(out))
    return out


def igemm_s4s8_packed(a, b_packed, scales, group, m, k, n):
    out = np.empty(m * n, np.float32)
    lib.oracle_igemm_s4s8_packed(_p(_c(a, np.int8)), _p(_c(b_packed, np.uint8)),
                                 _p(_c(scales, np.float32)), group, m, k, n, _p(out))
    return out


def quantize_row_i8(x, ties_even=False):
    x = _c(x, np.float32)
    q = np.empty(x.size, np.int8)
    f = lib.oracle_quantize_row_i8_te if ties_even else lib.oracle_quantize_row_i8
    s = f(_p(x), x.size, _p(q))
    return q, np.float32(s)


def quantize_int8_weights(w):
    w = _c(w, np.float32)
    n, k = w.shape
    q = np.empty((n, k), np.int8)
    s = np.empty(n, np.float32)
    lib.oracle_quantize_int8_weights(_p(w), n, k, _p(q), _p(s))
    return q, s


def pack_int4(w, group):
    w = _c(w, np.float32)
    n, k = w.shape
    p = np.empty((n, k // 2), np.uint8)
    s = np.empty((n, k // group), np.float32)
    lib.oracle_pack_int4(_p(w), n, k, group, _p(p), _p(s))
    return p, s


def silu(x: float) -> float:
    return float(lib.oracle_silu(x))


def gemv_i8(x, w, ws):
    x, w, ws = _c(x, np.float32), _c(w, np.int8), _c(ws, np.float32)
    n, k = w.shape
    y = np.empty(n, np.float32)
    lib.oracle_gemv_i8(_p(x), _p(w), _p(ws), n, k, _p(y))
    return y


def expert_i8(x, gw, gs, uw, us, dw, ds):
    H = x.size
    I = gw.shape[0]
    y = np.empty(H, np.float32)
    lib.oracle_expert_i8(_p(_c(x, np.float32)), H, I, _p(_c(gw, np.int8)), _p(_c(gs, np.float32)),
                         _p(_c(uw, np.int8)), _p(_c(us, np.float32)), _p(_c(dw, np.int8)),
                         _p(_c(ds, np.float32)), _p(y))
    return y


def router_logits(x, gate):
    x, gate = _c(x, np.float32), _c(gate, np.float32)
    E, H = gate.shape
    out = np.empty(E, np.float32)
    lib.oracle_router_logits(_p(x), H, _p(gate), E, _p(out))
    return out


def route(x, gate, topk=6, norm_topk_prob=False, scaling=1.0):
    """Returns (rc, idx [n,topk], w [n,topk]); rc < 0 mirrors the reference's
    'no finite router score' error."""
    x, gate = _c(x, np.float32), _c(gate, np.float32)
    n, H = x.shape
    E = gate.shape[0]
    idx = np.zeros((n, topk), np.int32)
    w = np.zeros((n, topk), np.float32)
    rc = lib.oracle_route(_p(x), n, H, _p(gate), E, topk, int(norm_topk_prob), float(scaling),
                          _p(idx), _p(w))
    return rc, idx, w


class MoeOracle:
    """Oracle view of a synth.MoeWeightsHost (all experts must be present)."""

    def __init__(self, W, norm_topk_prob=True, scaling=1.0):
        self.W = W
        self._keep = []
        L = MoeLayerC()
        L.hidden, L.inter, L.n_experts, L.topk = W.hidden, W.inter, W.n_experts, W.topk
        L.shared_inter = W.shared_inter
        L.norm_topk_prob = int(norm_topk_prob)
        L.routed_scaling_factor = scaling
        L.group = W.group
        self._set(L, "router", W.router)
        for name, arr in W.arrays.items():
            self._set(L, name, arr)
        self.L = L

    def _set(self, L, name, arr):
        arr = np.ascontiguousarray(arr)
        self._keep.append(arr)
        setattr(L, name, arr.ctypes.data)

    def decode(self, x):
        x = _c(x, np.float32)
        m = x.shape[0]
        y = np.empty((m, self.W.hidden), np.float32)
        idx = np.empty((m, self.W.topk), np.int32)
        w = np.empty((m, self.W.topk), np.float32)
        rc = lib.oracle_moe_decode(C.byref(self.L), _p(x), m, _p(y), _p(idx), _p(w))
        return rc, y, idx, w

    def forward(self, x, idx, w):
        x = _c(x, np.float32)
        m = x.shape[0]
        y = np.empty((m, self.W.hidden), np.float32)
        rc = lib.oracle_moe_decode_routed(C.byref(self.L), _p(x), m, _p(_c(idx, np.int32)),
                                          _p(_c(w, np.float32)), _p(y))
        assert rc == 0, rc
        return y

    def prefill(self, x):
        """moe_block_i8 (decoder.rs:2142-2181): route, experts in ascending id
        (ties-even activation quantisation), then the shared expert."""
        x = _c(x, np.float32)
        m = x.shape[0]
        y = np.empty((m, self.W.hidden), np.float32)
        idx = np.empty((m, self.W.topk), np.int32)
        w = np.empty((m, self.W.topk), np.float32)
        rc = lib.oracle_moe_prefill(C.byref(self.L), _p(x), m, _p(y), _p(idx), _p(w))
        return rc, y, idx, w

    def prefill_routed(self, x, idx, w):
        x = _c(x, np.float32)
        m = x.shape[0]
        y = np.empty((m, self.W.hidden), np.float32)
        rc = lib.oracle_moe_prefill_routed(C.byref(self.L), _p(x), m, _p(_c(idx, np.int32)),
                                           _p(_c(w, np.float32)), _p(y))
        assert rc == 0, rc
        return y

    def cpu_forward(self, x, idx, w, threads):
        """The timed CPU baseline (restated AVX-512-VNNI tier + threaded driver)."""
        x = _c(x, np.float32)
        m = x.shape[0]
        y = np.empty((m, self.W.hidden), np.float32)
        rc = lib.oracle_cpu_moe_decode(C.byref(self.L), _p(x), m, _p(_c(idx, np.int32)),
                                       _p(_c(w, np.float32)), _p(y), threads)
        assert rc == 0, rc
        return y


def vocab_tile_ranges(n, tiles):
    t = max(1, min(tiles, max(n, 1)))
    s = np.empty(t, np.uint64)
    e = np.empty(t, np.uint64)
    lib.oracle_vocab_tile_ranges(n, tiles, _p(s), _p(e))
    return list(zip(s.tolist(), e.tolist()))


def argmax_row(v):
    v = _c(v, np.float32)
    return int(lib.oracle_argmax_row(_p(v), v.size))


def rms_norm(x, w=None, eps=1e-6):
    """nn.rs:240 rms_norm in the order this project defines (see focr_oracle.c)."""
    x = _c(x, np.float32)
    rows, cols = x.shape
    y = np.empty_like(x)
    lib.oracle_rms_norm(_p(x), rows, cols, _p(_c(w, np.float32)) if w is not None else None,
                        float(eps), _p(y))
    return y


def rope_table(positions, head_dim, theta=10000.0):
    """decoder.rs:171 RopeTable::build -> (cos, sin), each [seq, head_dim]."""
    pos = np.ascontiguousarray(np.asarray(positions, dtype=np.uintp))
    seq = pos.size
    cos_t = np.empty((seq, head_dim), np.float32)
    sin_t = np.empty((seq, head_dim), np.float32)
    lib.oracle_rope_table(pos.ctypes.data, seq, head_dim, float(theta), _p(cos_t), _p(sin_t))
    return cos_t, sin_t


def apply_rope(x, cos_t, sin_t, head_dim):
    """decoder.rs:229 apply_rope, returning a rotated copy."""
    y = np.array(_c(x, np.float32), copy=True)
    seq, cols = y.shape
    lib.oracle_apply_rope(_p(y), seq, cols, head_dim, _p(_c(cos_t, np.float32)),
                          _p(_c(sin_t, np.float32)))
    return y


def attention_decode(q, ref_k, ref_v, prefill_len, ring_k, ring_v, ring_len):
    """rswa.rs:894 decode_attention_scalar (online-softmax fold)."""
    q = _c(q, np.float32)
    heads, hd = q.shape
    out = np.empty_like(q)
    rc = lib.oracle_attention_decode(_p(q), _p(_c(ref_k, np.float32)), _p(_c(ref_v, np.float32)),
                                     prefill_len, ref_k.shape[1], _p(_c(ring_k, np.float32)),
                                     _p(_c(ring_v, np.float32)), ring_len, ring_k.shape[1],
                                     heads, hd, _p(out))
    assert rc == 0, rc
    return out


def linear_i8(x, w, ws, ties_even, threads=0):
    """nn::linear_int8_dynamic (ties_even) / gemv_i8 (half away), row by row;
    threads > 0 runs the restated dispatched tier (same values)."""
    x, w, ws = _c(x, np.float32), _c(w, np.int8), _c(ws, np.float32)
    m, k = x.shape
    n = w.shape[0]
    y = np.empty((m, n), np.float32)
    if threads > 0:
        lib.oracle_cpu_linear_i8(_p(x), m, k, _p(w), _p(ws), n, int(ties_even), _p(y), threads)
    else:
        lib.oracle_linear_i8(_p(x), m, k, _p(w), _p(ws), n, int(ties_even), _p(y))
    return y


def swiglu_mlp_i8(x, d, ties_even):
    """The dense layer-0 MLP (decoder.rs:1711 / :2120) with d = gate/up/down _w/_s."""
    x = _c(x, np.float32)
    m, H = x.shape
    I = d["gate_w"].shape[0]
    a = {k: _c(v, np.int8 if k.endswith("_w") else np.float32) for k, v in d.items()}
    y = np.empty((m, H), np.float32)
    lib.oracle_swiglu_mlp_i8(_p(x), m, H, I, _p(a["gate_w"]), _p(a["gate_s"]), _p(a["up_w"]),
                             _p(a["up_s"]), _p(a["down_w"]), _p(a["down_s"]), int(ties_even),
                             _p(y))
    return y


def attention_prefill(q, k, v, heads, head_dim=128):
    q, k, v = _c(q, np.float32), _c(k, np.float32), _c(v, np.float32)
    out = np.empty_like(q)
    rc = lib.oracle_attention_prefill(_p(q), _p(k), _p(v), q.shape[0], heads, head_dim, _p(out))
    assert rc == 0, rc
    return out


class DecoderOracle:
    """CPU restatement of the int8 decoder loop over a synth.decoder_model:
    prefill_with_cache_i8 (decoder.rs:2412-2540), decode_step_with_cache_i8
    (:2542-2640), lm_head_cached_i8 (:2275) + argmax_row, and the greedy loop
    of generate_cached_i8 (native_engine/mod.rs:1860-1898), with the RingCache
    slot rule of rswa.rs:451-500."""

    HD, WINDOW, EPS = 128, 128, 1e-6

    def __init__(self, W, threads=0):
        """threads > 0: decode steps run the projections, the dense MLP, the
        MoE experts and the lm-head on the restated dispatched tier
        (cpu_baseline.c, same values) -- the timed CPU baseline."""
        self.W = W
        self.threads = threads
        self.D = W.heads * self.HD
        self.moe = [MoeOracle(L.moe, norm_topk_prob=W.norm_topk_prob,
                              scaling=W.routed_scaling_factor) if L.moe is not None else None
                    for L in W.layers]

    def _heads(self, t):  # [seq, D] -> [heads, seq, HD]
        return np.ascontiguousarray(t.reshape(t.shape[0], self.W.heads, self.HD).transpose(1, 0, 2))

    def prefill(self, x):
        x = _c(x, np.float32)
        seq = x.shape[0]
        cos_t, sin_t = rope_table(np.arange(seq), self.HD)
        self.ref, self.ring = [], []
        for li, L in enumerate(self.W.layers):
            P = L.proj
            n = rms_norm(x, L.input_ln, self.EPS)
            q = apply_rope(linear_i8(n, P["q_w"], P["q_s"], True), cos_t, sin_t, self.HD)
            k = apply_rope(linear_i8(n, P["k_w"], P["k_s"], True), cos_t, sin_t, self.HD)
            v = linear_i8(n, P["v_w"], P["v_s"], True)
            self.ref.append((self._heads(k), self._heads(v)))
            z = np.zeros((self.W.heads, self.WINDOW, self.HD), np.float32)
            self.ring.append((z, z.copy()))
            ctx = attention_prefill(q, k, v, self.W.heads, self.HD)
            h = x + linear_i8(ctx, P["o_w"], P["o_s"], True)
            n2 = rms_norm(h, L.post_ln, self.EPS)
            if L.moe is not None:
                rc, mlp, _, _ = self.moe[li].prefill(n2)
                assert rc == 0, rc
            else:
                mlp = swiglu_mlp_i8(n2, L.dense, True)
            x = h + mlp
        self.prefill_len, self.ring_len, self.ring_pos = seq, 0, 0
        return x

    def decode_step(self, x, position):
        x = _c(x, np.float32).reshape(1, -1)
        cos_t, sin_t = rope_table([position], self.HD)
        if self.ring_len < self.WINDOW:
            slot = self.ring_len
            self.ring_len += 1
            self.ring_pos = self.ring_len % self.WINDOW
        else:
            slot = self.ring_pos
            self.ring_pos = (self.ring_pos + 1) % self.WINDOW
        for li, L in enumerate(self.W.layers):
            P = L.proj
            n = rms_norm(x, L.input_ln, self.EPS)
            th = self.threads
            q = apply_rope(linear_i8(n, P["q_w"], P["q_s"], False, th), cos_t, sin_t, self.HD)
            k = apply_rope(linear_i8(n, P["k_w"], P["k_s"], False, th), cos_t, sin_t, self.HD)
            v = linear_i8(n, P["v_w"], P["v_s"], False, th)
            rk, rv = self.ring[li]
            rk[:, slot] = k.reshape(self.W.heads, self.HD)
            rv[:, slot] = v.reshape(self.W.heads, self.HD)
            fk, fv = self.ref[li]
            ctx = attention_decode(q.reshape(self.W.heads, self.HD), fk, fv, self.prefill_len,
                                   rk, rv, self.ring_len)
            h = x + linear_i8(ctx.reshape(1, -1), P["o_w"], P["o_s"], False, th)
            n2 = rms_norm(h, L.post_ln, self.EPS)
            if L.moe is not None and th:
                M = L.moe
                rc, idx, w = route(n2, M.router, M.topk, self.W.norm_topk_prob,
                                   self.W.routed_scaling_factor)
                assert rc == 0, rc
                mlp = self.moe[li].cpu_forward(n2, idx, w, th)
            elif L.moe is not None:
                rc, mlp, _, _ = self.moe[li].decode(n2)
                assert rc == 0, rc
            elif th:
                d = L.dense
                g = linear_i8(n2, d["gate_w"], d["gate_s"], False, th)
                u = linear_i8(n2, d["up_w"], d["up_s"], False, th)
                act = np.empty_like(g)
                lib.oracle_silu_mul(_p(g), _p(u), g.size, _p(act))
                mlp = linear_i8(act, d["down_w"], d["down_s"], False, th)
            else:
                mlp = swiglu_mlp_i8(n2, L.dense, False)
            x = h + mlp
        return x

    def lm_head(self, row):
        n = rms_norm(_c(row, np.float32).reshape(1, -1), self.W.final_norm, self.EPS)
        return linear_i8(n, self.W.lm_w, self.W.lm_s, False, self.threads)[0]

    def generate(self, embeds, n_tokens, hiddens=None):
        h = self.prefill(embeds)
        seq = embeds.shape[0]
        out = []
        for i in range(n_tokens):
            if hiddens is not None:
                hiddens.append(h[-1].copy())
            tok = argmax_row(self.lm_head(h[-1]))
            out.append(tok)
            if i + 1 == n_tokens:
                break
            h = self.decode_step(self.W.embed[tok], seq + i)
        return np.array(out, np.int64)


def ep_dispatch_layout(idx, e_local, world, cap):
    """Host restatement of the expert-parallel dispatch layout (the library's
    ep_dispatch_kernel): pair b = t*topk + j with expert e >= 0 goes to owner
    d = e // e_local, at position pos = number of earlier pairs (in b order)
    with the same owner; its partial comes back to return row d*cap + pos.
    Returns (rows [P] (-1 = empty slot), per-owner lists of (pos, b))."""
    flat = np.asarray(idx, np.int64).reshape(-1)
    rows = np.full(flat.size, -1, np.int64)
    sends = [[] for _ in range(world)]
    for b, e in enumerate(flat):
        if e < 0:
            continue
        d = int(e) // e_local
        pos = len(sends[d])
        assert pos < cap
        sends[d].append((pos, b))
        rows[b] = d * cap + pos
    return rows, sends
