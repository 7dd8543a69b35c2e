"""``.focrq`` reader/writer (CPU).

The first group restates the reference loader's own unit tests
(src/native_engine/weights.rs:1229-1380) on hand-assembled blobs whose header
JSON is written the way those tests write it (unsorted keys); the rest cover
the format document's validation rules, writer determinism and the mapping
onto the MoE layer / lm-head arrays the GPU engine consumes.
"""
import json
import struct

import numpy as np
import pytest

from franken_ocr_b200 import focrq, synth
from franken_ocr_b200.focrq import FormatMismatch, Weights
from franken_ocr_b200.quant import quantize_int8_f32

NOTICE = focrq.MODEL_LICENSE_NOTICE


def blob(directory: str = "{}", payload: bytes = b"", version: int = 1, arch: int = 0,
         sha: bytes = bytes(32), notice: str = NOTICE, header_sha: str = "",
         model_id: str | None = None) -> bytes:
    """A hand-assembled blob in the reference tests' layout
    (weights.rs:1085-1180)."""
    h = (f'{{"tensors":{directory},"arch_target":{arch},"source_sha256":{json.dumps(header_sha)},'
         f'"license_notice":{json.dumps(notice)}')
    if model_id is not None:
        h += f',"model_id":{json.dumps(model_id)}'
    h = (h + "}").encode()
    return (b"FOCRQ\0" + struct.pack("<IB", version, arch) + sha + struct.pack("<Q", len(h)) + h
            + payload)


def bf16_bytes(vals):
    return (np.asarray(vals, np.float32).view(np.uint32) >> 16).astype("<u2").tobytes()


# -- ported reference loader tests ---------------------------------------------
def test_roundtrips_bf16_tensor_bit_exactly():
    vals = [1.0, -2.0, 0.5, 3.0, 0.0, -0.25]
    p = bf16_bytes(vals)
    d = f'{{"w":{{"dtype":"BF16","shape":[2,3],"byte_offset":0,"byte_len":{len(p)}}}}}'
    w = Weights.from_bytes(blob(d, p, arch=2, sha=bytes([7]) * 32))
    assert len(w) == 1 and w.arch_target == 2
    assert w.source_sha256 == "07" * 32
    assert w.license_notice == NOTICE
    assert w.record("w").dtype == "BF16" and w.record("w").shape == (2, 3)
    m = w.mat("w")
    assert m.shape == (2, 3) and m.dtype == np.float32
    assert np.array_equal(m.ravel(), np.asarray(vals, np.float32))


def test_rejects_without_baidu_mit_license_notice():
    with pytest.raises(FormatMismatch, match="license_notice.*MIT License"):
        Weights.from_bytes(blob(notice="Copyright (c) 2026 Baidu"))


def test_absent_model_id_resolves_to_unlimited_ocr():
    assert Weights.from_bytes(blob()).model_id == "unlimited-ocr"


def test_empty_model_id_resolves_to_unlimited_ocr():
    assert Weights.from_bytes(blob(model_id="")).model_id == "unlimited-ocr"


def test_got_ocr2_with_apache_notice_loads():
    w = Weights.from_bytes(blob(notice="GOT-OCR2.0 (StepFun) - Apache-2.0", model_id="got-ocr2"))
    assert w.model_id == "got-ocr2"


def test_unknown_model_id_is_refused():
    with pytest.raises(FormatMismatch, match="unknown model_id"):
        Weights.from_bytes(blob(model_id="not-a-model"))


def test_got_ocr2_with_wrong_notice_is_refused():
    with pytest.raises(FormatMismatch, match="does not match the registered got-ocr2 notice"):
        Weights.from_bytes(blob(model_id="got-ocr2"))


def test_header_source_sha256_overrides_prefix_when_valid():
    good = "ab" * 32
    w = Weights.from_bytes(blob(sha=bytes([1]) * 32, header_sha=good))
    assert w.source_sha256 == good
    # header arch_target 0 defers to the prefix byte
    assert Weights.from_bytes(blob(arch=0)).arch_target == 0


@pytest.mark.parametrize("bad", ["AB" * 32, "ab" * 31, "zz" * 32])
def test_rejects_malformed_header_source_sha256(bad):
    with pytest.raises(FormatMismatch, match="source_sha256"):
        Weights.from_bytes(blob(header_sha=bad))


# -- prefix / header structure ----------------------------------------------------
def test_rejects_newer_format_version():
    with pytest.raises(FormatMismatch, match="format_version 2"):
        Weights.from_bytes(blob(version=2))


def test_rejects_bad_magic_and_truncation():
    b = bytearray(blob())
    b[0:6] = b"FOCRX\0"
    with pytest.raises(FormatMismatch, match="magic"):
        Weights.from_bytes(bytes(b))
    with pytest.raises(FormatMismatch, match="truncated"):
        Weights.from_bytes(blob()[:50])


def test_rejects_header_overrun_and_bad_json():
    b = blob()
    cut = b[:-3]
    with pytest.raises(FormatMismatch, match="overruns"):
        Weights.from_bytes(cut)
    h = b"{not json"
    bad = b"FOCRQ\0" + struct.pack("<IB", 1, 0) + bytes(32) + struct.pack("<Q", len(h)) + h
    with pytest.raises(FormatMismatch, match="JSON invalid"):
        Weights.from_bytes(bad)
    with pytest.raises(FormatMismatch, match="JSON invalid"):
        Weights.from_bytes(blob(directory="[]"))


def test_missing_file_is_model_not_found(tmp_path):
    with pytest.raises(focrq.ModelNotFound):
        Weights.load(tmp_path / "nope.focrq")


# -- directory validation ------------------------------------------------------------
def rec(**kw):
    return json.dumps({"x": kw})


def test_rejects_range_past_payload():
    with pytest.raises(FormatMismatch, match="payload is 8 bytes"):
        Weights.from_bytes(blob(rec(dtype="F32", shape=[4], byte_offset=0, byte_len=16),
                                bytes(8)))


def test_rejects_byte_len_shape_mismatch():
    with pytest.raises(FormatMismatch, match="byte_len 8 != shape x dtype 16"):
        Weights.from_bytes(blob(rec(dtype="F32", shape=[4], byte_offset=0, byte_len=8),
                                bytes(16)))


def test_rejects_unknown_dtype_and_negative_fields():
    with pytest.raises(FormatMismatch, match="unknown dtype"):
        Weights.from_bytes(blob(rec(dtype="I8", shape=[4], byte_offset=0, byte_len=4), bytes(4)))
    with pytest.raises(FormatMismatch, match="non-negative"):
        Weights.from_bytes(blob(rec(dtype="F32", shape=[1], byte_offset=-4, byte_len=4),
                                bytes(4)))


def test_qint8_scale_count_and_group_rules():
    ok = dict(dtype="QInt8PerChan", shape=[2, 4], byte_offset=0, byte_len=8, scales_offset=64,
              scales_len=8, group_size=0, tier=0)
    w = Weights.from_bytes(blob(rec(**ok), bytes(72)))
    q, s = w.qint8("x")
    assert q.shape == (2, 4) and s.shape == (2,)
    with pytest.raises(FormatMismatch, match="scales_len == n"):
        Weights.from_bytes(blob(rec(**{**ok, "scales_len": 4}), bytes(72)))
    with pytest.raises(FormatMismatch, match="group_size must be 0"):
        Weights.from_bytes(blob(rec(**{**ok, "group_size": 16}), bytes(72)))


def test_qint4_group_rules():
    ok = dict(dtype="QInt4PerGroup", shape=[2, 32], byte_offset=0, byte_len=32,
              scales_offset=64, scales_len=8, group_size=32, tier=3)
    w = Weights.from_bytes(blob(rec(**ok), bytes(72)))
    p, s, g = w.qint4("x")
    assert p.shape == (2, 16) and s.shape == (2, 1) and g == 32
    assert w.record("x").tier == 3
    with pytest.raises(FormatMismatch, match="must be 16 or 32"):
        Weights.from_bytes(blob(rec(**{**ok, "group_size": 8}), bytes(72)))
    with pytest.raises(FormatMismatch, match="n \\* \\(k / group_size\\)"):
        Weights.from_bytes(blob(rec(**{**ok, "group_size": 16}), bytes(72)))
    with pytest.raises(FormatMismatch, match="odd element count"):
        Weights.from_bytes(blob(rec(**{**ok, "shape": [1, 33], "byte_len": 16}), bytes(72)))


def test_rejects_overlapping_ranges():
    d = json.dumps({"a": dict(dtype="F32", shape=[4], byte_offset=0, byte_len=16),
                    "b": dict(dtype="F32", shape=[4], byte_offset=8, byte_len=16)})
    with pytest.raises(FormatMismatch, match="overlap"):
        Weights.from_bytes(blob(d, bytes(32)))


def test_accessor_type_errors():
    p = bf16_bytes([1.0, 2.0])
    w = Weights.from_bytes(blob(rec(dtype="BF16", shape=[1, 2], byte_offset=0, byte_len=4), p))
    with pytest.raises(FormatMismatch, match="not QInt8PerChan"):
        w.qint8("x")
    with pytest.raises(FormatMismatch, match="not QInt4PerGroup"):
        w.qint4("x")
    with pytest.raises(FormatMismatch, match="not found"):
        w.mat("y")
    # a high-precision record goes through the per-row quantiser
    q, s = w.int8_rows("x")
    q2, s2 = quantize_int8_f32(np.array([[1.0, 2.0]], np.float32))
    assert np.array_equal(q, q2) and np.array_equal(s, s2)


def test_f16_widening_is_exact():
    vals = np.array([0.5, -1.25, 65504.0, 2.0 ** -24], np.float16)
    p = vals.astype("<f2").tobytes()
    w = Weights.from_bytes(blob(rec(dtype="F16", shape=[4], byte_offset=0, byte_len=8), p))
    assert np.array_equal(w.mat("x"), vals.astype(np.float32))


# -- writer -----------------------------------------------------------------------------
def small_layer(group=0, shared=64):
    return synth.moe_layer(77, hidden=64, inter=32, n_experts=8, topk=2, shared_inter=shared,
                           group=group)


def test_writer_is_deterministic_and_reloads_byte_identically():
    W = small_layer()
    a = focrq.Writer(source_sha256=focrq.sha256_bytes(b"src"))
    focrq.write_moe_layer(a, 3, W)
    b1 = a.to_bytes()
    assert b1 == a.to_bytes()
    w = Weights.from_bytes(b1)
    # convert -> load -> reserialise is byte-identical
    r = focrq.Writer(source_sha256=bytes.fromhex(w.source_sha256))
    focrq.write_moe_layer(r, 3, focrq.moe_layer_weights(w, 3, topk=2))
    assert r.to_bytes() == b1


def test_writer_alignment_and_zero_padding():
    W = small_layer(group=16)
    wr = focrq.Writer()
    focrq.write_moe_layer(wr, 0, W)
    b = wr.to_bytes()
    w = Weights.from_bytes(b)
    (hl,) = struct.unpack_from("<Q", b, 43)
    hdr = json.loads(b[51:51 + hl])
    assert list(hdr) == sorted(hdr) and list(hdr["tensors"]) == sorted(hdr["tensors"])
    assert b[51:51 + hl] == json.dumps(hdr, sort_keys=True, separators=(",", ":")).encode()
    used = np.zeros(len(b) - w.payload_base, bool)
    for r in w.directory.values():
        assert r.byte_offset % 64 == 0
        used[r.byte_offset:r.byte_offset + r.byte_len] = True
        if r.scales_len:
            assert r.scales_offset % 64 == 0
            used[r.scales_offset:r.scales_offset + r.scales_len] = True
    pay = np.frombuffer(b, np.uint8)[w.payload_base:]
    assert not pay[~used].any()


# -- model mapping ----------------------------------------------------------------------
@pytest.mark.parametrize("group,shared", [(0, 64), (0, 0), (16, 64), (32, 0)])
def test_moe_layer_roundtrip(group, shared):
    W = small_layer(group, shared)
    wr = focrq.Writer()
    focrq.write_moe_layer(wr, 5, W)
    w = Weights.from_bytes(wr.to_bytes())
    w.census(focrq.moe_tensor_names(5, 8, shared=bool(shared)))
    L = focrq.moe_layer_weights(w, 5, topk=2)
    assert (L.hidden, L.inter, L.n_experts, L.shared_inter, L.group) == (64, 32, 8, shared, group)
    assert np.array_equal(L.router, W.router)
    assert sorted(L.arrays) == sorted(W.arrays)
    for k in W.arrays:
        assert np.array_equal(L.arrays[k], W.arrays[k]), k


def test_moe_layer_expert_range_for_one_rank():
    W = small_layer()
    wr = focrq.Writer()
    focrq.write_moe_layer(wr, 0, W)
    w = Weights.from_bytes(wr.to_bytes())
    L = focrq.moe_layer_weights(w, 0, topk=2, expert_begin=4, expert_count=4)
    assert (L.expert_begin, L.expert_count) == (4, 4)
    assert np.array_equal(L.arrays["gate_w"], W.arrays["gate_w"][4:])
    with pytest.raises(ValueError):
        focrq.moe_layer_weights(w, 0, expert_begin=6, expert_count=4)
    with pytest.raises(FormatMismatch, match="not found"):
        focrq.moe_layer_weights(w, 1)


def test_high_precision_experts_are_quantised_at_load():
    """quant_oc_loaded: BF16 expert records are widened and quantised per row,
    identical to quantising the same f32 values directly."""
    g = np.random.default_rng(5)
    wr = focrq.Writer()
    p = focrq.layer_prefix(0)
    wr.add_bf16(f"{p}.gate.weight", g.standard_normal((4, 32), dtype=np.float32))
    mats = {}
    for e in range(4):
        for r, shp in (("gate", (16, 32)), ("up", (16, 32)), ("down", (32, 16))):
            a = g.standard_normal(shp, dtype=np.float32) * np.float32(0.02)
            a = ((a.view(np.uint32) >> 16) << 16).view(np.float32)  # bf16-exact
            mats[(e, r)] = a
            wr.add_bf16(f"{p}.experts.{e}.{r}_proj.weight", a)
    L = focrq.moe_layer_weights(Weights.from_bytes(wr.to_bytes()), 0, topk=2)
    for e in range(4):
        for r in ("gate", "up", "down"):
            q, s = quantize_int8_f32(mats[(e, r)])
            assert np.array_equal(L.arrays[r + "_w"][e], q)
            assert np.array_equal(L.arrays[r + "_s"][e], s)
    assert L.shared_inter == 0


def test_mixed_expert_storage_is_refused():
    W = small_layer(shared=0)
    wr = focrq.Writer()
    focrq.write_moe_layer(wr, 0, W)
    W4 = small_layer(group=16, shared=0)
    p = focrq.layer_prefix(0)
    wr.add_qint4(f"{p}.experts.0.gate_proj.weight", W4.arrays["gate_p"][0],
                 W4.arrays["gate_gs"][0], 16)
    with pytest.raises(FormatMismatch, match="mix"):
        focrq.moe_layer_weights(Weights.from_bytes(wr.to_bytes()), 0)


def test_lm_head_shard_rows():
    q, s = synth.lm_head(3, 200, hidden=64, block=64)
    wr = focrq.Writer()
    wr.add_qint8("lm_head.weight", q, s)
    w = Weights.from_bytes(wr.to_bytes())
    q1, s1 = focrq.lm_head_weights(w, 50, 100)
    assert np.array_equal(q1, q[50:150]) and np.array_equal(s1, s[50:150])
    with pytest.raises(ValueError):
        focrq.lm_head_weights(w, 150, 100)


def test_decoder_roundtrip_through_focrq():
    """A whole synthetic decoder written under the canonical names reloads
    into identical arrays (and into the oracle decoder's identical tokens)."""
    from oracle import oracle as O

    W = synth.decoder_model(9, layers=3, n_experts=4, topk=2, dense_inter=128, vocab=256,
                            shared_inter=64)
    wr = focrq.Writer()
    focrq.write_decoder(wr, W)
    w = Weights.from_bytes(wr.to_bytes())
    w.census(focrq.decoder_tensor_names(3, 4))
    R = focrq.decoder_weights(w, topk=2)
    assert (R.hidden, R.heads, R.vocab, len(R.layers)) == (W.hidden, W.heads, W.vocab, 3)
    for a, b in ((R.embed, W.embed), (R.final_norm, W.final_norm), (R.lm_w, W.lm_w),
                 (R.lm_s, W.lm_s)):
        assert np.array_equal(a, b)
    for La, Lb in zip(R.layers, W.layers):
        assert np.array_equal(La.input_ln, Lb.input_ln) and np.array_equal(La.post_ln, Lb.post_ln)
        for k in Lb.proj:
            assert np.array_equal(La.proj[k], Lb.proj[k]), k
        if Lb.dense is not None:
            for k in Lb.dense:
                assert np.array_equal(La.dense[k], Lb.dense[k]), k
        else:
            for k in Lb.moe.arrays:
                assert np.array_equal(La.moe.arrays[k], Lb.moe.arrays[k]), k
    e = synth.prompt_embeds(9, 5, W.hidden)
    assert np.array_equal(O.DecoderOracle(R).generate(e, 4), O.DecoderOracle(W).generate(e, 4))


def test_decoder_weights_rejects_bad_shapes():
    W = synth.decoder_model(9, layers=1, dense_inter=128, vocab=64)
    W.layers[0].proj["o_w"] = W.layers[0].proj["o_w"][:, :640].copy()
    wr = focrq.Writer()
    focrq.write_decoder(wr, W)
    with pytest.raises(FormatMismatch, match="o_proj"):
        focrq.decoder_weights(Weights.from_bytes(wr.to_bytes()))


# -- golden fixtures from the reference (tests/golden/make_golden.py) -----------------
GOLDEN = __import__("pathlib").Path(__file__).resolve().parent / "golden"


def test_registry_matches_the_reference_registry():
    want = json.loads((GOLDEN / "model_registry.json").read_text())
    assert focrq.MODEL_REGISTRY == want
    assert focrq.MODEL_LICENSE_NOTICE == want["unlimited-ocr"]


def test_reference_minimal_header_example_loads():
    """The format document's minimal header, as a writer would emit it
    (canonical JSON), loads with an empty directory and keeps its metadata."""
    hdr = json.loads((GOLDEN / "focrq_minimal_header.json").read_text())
    hj = json.dumps(hdr, sort_keys=True, separators=(",", ":")).encode()
    b = (b"FOCRQ\0" + struct.pack("<IB", hdr["format_version"], hdr["arch_target"]) + bytes(32)
         + struct.pack("<Q", len(hj)) + hj)
    w = Weights.from_bytes(b)
    assert len(w) == 0 and w.model_id == "unlimited-ocr" and w.arch_target == 0
    assert w.source_sha256 == "0" * 64
    assert w.header["model_config"]["hidden_size"] == 1280
    assert w.header["packing_manifest"]["rounding"] == "round_ties_to_even"


def test_decoder_model_config_must_match_the_tensors():
    W = synth.decoder_model(9, layers=1, dense_inter=128, vocab=64)
    good = {"hidden_size": 1280, "num_attention_heads": 10, "num_hidden_layers": 1,
            "vocab_size": 64}
    wr = focrq.Writer(model_config=good)
    focrq.write_decoder(wr, W)
    focrq.decoder_weights(Weights.from_bytes(wr.to_bytes()))
    wr = focrq.Writer(model_config={**good, "num_hidden_layers": 12})
    focrq.write_decoder(wr, W)
    with pytest.raises(FormatMismatch, match="num_hidden_layers"):
        focrq.decoder_weights(Weights.from_bytes(wr.to_bytes()))


def test_decoder_layer_prefix_and_heads_from_model_config():
    """Loading a prefix of the layers is valid with a matching model_config;
    heads come from model_config, and an explicit disagreeing value is a
    mismatch."""
    W = synth.decoder_model(9, layers=2, dense_inter=128, vocab=64)
    cfg = {"hidden_size": 1280, "num_attention_heads": 10, "num_hidden_layers": 2,
           "vocab_size": 64}
    wr = focrq.Writer(model_config=cfg)
    focrq.write_decoder(wr, W)
    w = Weights.from_bytes(wr.to_bytes())
    D = focrq.decoder_weights(w, n_layers=1)
    assert len(D.layers) == 1 and D.heads == 10
    with pytest.raises(FormatMismatch, match="num_attention_heads"):
        focrq.decoder_weights(w, heads=5)
