"""``.focrq`` weight container: reader, validator and a deterministic writer,
plus the mapping from its tensor directory onto the GPU MoE layer and lm-head.

The reader follows the reference loader ``Weights::from_focrq_bytes``
(src/native_engine/weights.rs:462-544) and the format document
(docs/focrq-format.md, "Loader Algorithm"):

* fixed 51-byte little-endian prefix ``magic[6]="FOCRQ\\0" | format_version u32
  | arch_target u8 | source_sha256[32] | header_len u64``; a version above 1
  is refused;
* the header is a JSON object whose ``tensors`` map names byte ranges relative
  to the payload, which starts right after the header;
* ``model_id`` (absent or empty = ``unlimited-ocr``) must be in the registry
  (model_arch.rs:429-443), and ``license_notice`` must be the Baidu MIT
  notice for the default architecture or equal the registered notice for any
  other (weights.rs:97-121);
* every record's byte range and scale range lie inside the payload and its
  ``byte_len`` equals ``shape x dtype`` (weights.rs:949-987).

Every structural problem raises :class:`FormatMismatch`; a missing file
raises :class:`ModelNotFound` (the reference's exit 7 / exit 3).

Accessors mirror the reference's: :meth:`Weights.mat` widens F32/F16/BF16 to
f32 exactly (weights.rs:989-1023), :meth:`Weights.qint8` returns the int8
rows and per-row scales (weights.rs:821-857), :meth:`Weights.qint4` the packed
nibbles (low nibble = even column) and per-group scales (weights.rs:866-923).

:func:`moe_layer_weights` assembles one decoder layer's MoE weights under the
reference's canonical names (decoder.rs:2057-2092): ``model.layers.{l}.mlp.gate
.weight`` (router, high precision), ``...experts.{e}.{gate,up,down}_proj
.weight`` and ``...shared_experts.{gate,up,down}_proj.weight``.  A
``QInt8PerChan`` record is used verbatim and a high-precision one is quantised
per row at load time, the ``quant_oc_loaded`` rule (decoder.rs:1777-1786).
``QInt4PerGroup`` experts feed the int4 expert kernels directly.
:func:`decoder_weights` assembles the whole int8 decoder (norms, attention
projections, dense / MoE MLPs, final norm, lm-head, token embeddings) for the
device decoder (DecoderWeightCacheI8::build, decoder.rs:2018-2117).
"""
from __future__ import annotations

import hashlib
import json
import os
import struct
from dataclasses import dataclass

import numpy as np

from .quant import quantize_int8_f32
from .synth import MoeWeightsHost

MAGIC = b"FOCRQ\0"
FORMAT_VERSION = 1
PREFIX_LEN = 6 + 4 + 1 + 32 + 8
ALIGN = 64

ARCH_TARGETS = {0: "Generic", 1: "Aarch64Smmla", 2: "X86Vnni", 3: "X86Amx"}
DTYPES = ("F32", "F16", "BF16", "QInt8PerChan", "QInt4PerGroup")
GROUP_SIZES = (16, 32)

DEFAULT_MODEL_ID = "unlimited-ocr"
MODEL_LICENSE_NOTICE = "Baidu Unlimited-OCR - Copyright (c) 2026 Baidu, MIT License"
# Architecture registry: id -> the notice its artifacts must carry
# (src/native_engine/model_arch.rs:180-425).
MODEL_REGISTRY = {
    "unlimited-ocr": MODEL_LICENSE_NOTICE,
    "got-ocr2": "GOT-OCR2.0 (StepFun) - Apache-2.0",
    "smolvlm2": "SmolVLM2 (HuggingFaceTB) - Apache-2.0",
    "onechart": "OneChart - Apache-2.0",
    "tromr": "Polyphonic-TrOMR (NetEase) - Apache-2.0",
    "trocr": "TrOCR (Microsoft) - MIT",
    "pix2tex": "pix2tex / LaTeX-OCR - MIT",
}


class FormatMismatch(ValueError):
    """A blob that is not a loadable ``.focrq`` (exit 7 in the reference CLI)."""


class ModelNotFound(FileNotFoundError):
    """The weights file cannot be read (exit 3 in the reference CLI)."""


@dataclass(frozen=True)
class TensorRecord:
    """One directory entry (weights.rs:200-219); offsets are payload-relative."""
    dtype: str
    shape: tuple
    byte_offset: int
    byte_len: int
    scales_offset: int = 0
    scales_len: int = 0
    group_size: int = 0
    tier: int = 0

    def numel(self) -> int:
        n = 1
        for d in self.shape:
            n *= d
        return n

    def expected_byte_len(self, name: str) -> int:
        n = self.numel()
        if self.dtype == "QInt4PerGroup":
            if n % 2:
                raise FormatMismatch(f"tensor {name!r}: QInt4 shape {list(self.shape)} has odd "
                                     f"element count {n}")
            return n // 2
        return n * {"F32": 4, "F16": 2, "BF16": 2, "QInt8PerChan": 1}[self.dtype]


def _uint(v, name: str, field: str) -> int:
    # JSON integers only (bool is an int subclass in Python; the reference's
    # serde rejects it).
    if isinstance(v, bool) or not isinstance(v, int) or v < 0:
        raise FormatMismatch(f"tensor {name!r}: {field} must be a non-negative integer")
    return v


def _parse_record(name: str, r) -> TensorRecord:
    if not isinstance(r, dict):
        raise FormatMismatch(f"tensor {name!r}: record is not an object")
    for f in ("dtype", "shape", "byte_offset", "byte_len"):
        if f not in r:
            raise FormatMismatch(f"tensor {name!r}: missing field {f!r}")
    if r["dtype"] not in DTYPES:
        raise FormatMismatch(f"tensor {name!r}: unknown dtype {r['dtype']!r}")
    if not isinstance(r["shape"], list):
        raise FormatMismatch(f"tensor {name!r}: shape must be an array")
    shape = tuple(_uint(d, name, "shape") for d in r["shape"])
    tier = _uint(r.get("tier", 0), name, "tier")
    if tier > 255:
        raise FormatMismatch(f"tensor {name!r}: tier {tier} exceeds u8")
    return TensorRecord(r["dtype"], shape, _uint(r["byte_offset"], name, "byte_offset"),
                        _uint(r["byte_len"], name, "byte_len"),
                        _uint(r.get("scales_offset", 0), name, "scales_offset"),
                        _uint(r.get("scales_len", 0), name, "scales_len"),
                        _uint(r.get("group_size", 0), name, "group_size"), tier)


def resolve_model_id(declared: str) -> str:
    """weights.rs:71-83: empty = default; unknown non-empty ids are refused."""
    if not declared:
        return DEFAULT_MODEL_ID
    if declared not in MODEL_REGISTRY:
        raise FormatMismatch(f".focrq declares unknown model_id {declared!r} (not in the model "
                             "registry; this build cannot load it)")
    return declared


def validate_license_notice(notice: str, model_id: str) -> None:
    """weights.rs:97-121."""
    if model_id == DEFAULT_MODEL_ID:
        if notice == MODEL_LICENSE_NOTICE or ("Copyright (c) 2026 Baidu" in notice
                                              and "MIT License" in notice):
            return
        raise FormatMismatch(".focrq license_notice must include Copyright (c) 2026 Baidu and "
                             "MIT License")
    expected = MODEL_REGISTRY[model_id]
    if notice != expected:
        raise FormatMismatch(f".focrq license_notice does not match the registered {model_id} "
                             f"notice (expected {expected!r})")


def _validate_sha_hex(s: str) -> None:
    if len(s) != 64 or any(c not in "0123456789abcdef" for c in s):
        raise FormatMismatch(".focrq source_sha256 must be 64 lowercase hex chars when present")


def validate_directory(directory: dict, payload_len: int) -> None:
    """weights.rs:949-987, plus the format document's quantised-record rules:
    scale counts, group sizes and non-overlapping ranges."""
    ranges = []
    for name, rec in directory.items():
        end = rec.byte_offset + rec.byte_len
        if end > payload_len:
            raise FormatMismatch(f"tensor {name!r} ends at {end} but payload is {payload_len} "
                                 "bytes")
        expected = rec.expected_byte_len(name)
        if rec.byte_len != expected:
            raise FormatMismatch(f"tensor {name!r}: byte_len {rec.byte_len} != shape x dtype "
                                 f"{expected} ({rec.dtype}, shape {list(rec.shape)})")
        send = rec.scales_offset + rec.scales_len
        if send > payload_len:
            raise FormatMismatch(f"tensor {name!r} scales end at {send} but payload is "
                                 f"{payload_len} bytes")
        if rec.dtype == "QInt8PerChan":
            if rec.group_size != 0:
                raise FormatMismatch(f"tensor {name!r}: QInt8PerChan group_size must be 0")
            if len(rec.shape) != 2 or rec.scales_len != rec.shape[0] * 4:
                raise FormatMismatch(f"tensor {name!r}: QInt8PerChan needs shape [n, k] and "
                                     "scales_len == n * 4")
        elif rec.dtype == "QInt4PerGroup":
            if rec.group_size not in GROUP_SIZES:
                raise FormatMismatch(f"tensor {name!r}: group_size {rec.group_size} must be 16 "
                                     "or 32")
            if len(rec.shape) != 2 or rec.shape[1] % rec.group_size:
                raise FormatMismatch(f"tensor {name!r}: QInt4PerGroup needs shape [n, k] with "
                                     "group_size dividing k")
            if rec.scales_len != rec.shape[0] * (rec.shape[1] // rec.group_size) * 4:
                raise FormatMismatch(f"tensor {name!r}: scales_len {rec.scales_len} != "
                                     "n * (k / group_size) * 4")
        if rec.byte_len:
            ranges.append((rec.byte_offset, end, name))
        if rec.scales_len:
            ranges.append((rec.scales_offset, send, name + " (scales)"))
    ranges.sort()
    for (a0, a1, an), (b0, b1, bn) in zip(ranges, ranges[1:]):
        if b0 < a1:
            raise FormatMismatch(f"payload ranges of {an!r} and {bn!r} overlap")


class Weights:
    """An indexed ``.focrq`` blob (the reference's ``Weights``)."""

    def __init__(self, blob: bytes, payload_base: int, directory: dict, arch_target: int,
                 source_sha256: str, license_notice: str, model_id: str, header: dict):
        self._blob = memoryview(blob)
        self.payload_base = payload_base
        self.directory = directory
        self.arch_target = arch_target
        self.source_sha256 = source_sha256
        self.license_notice = license_notice
        self.model_id = model_id
        self.header = header

    # -- loading ---------------------------------------------------------------
    @classmethod
    def load(cls, path) -> "Weights":
        """Map the file read-only (no copy of the payload) and index it."""
        import mmap

        try:
            with open(path, "rb") as f:
                size = os.fstat(f.fileno()).st_size
                blob = (mmap.mmap(f.fileno(), 0, access=mmap.ACCESS_READ) if size >= PREFIX_LEN
                        else f.read())
        except OSError as e:
            raise ModelNotFound(f"cannot read weights at {os.fspath(path)}: {e}") from e
        return cls.from_bytes(blob)

    @classmethod
    def from_bytes(cls, blob: bytes) -> "Weights":
        n = len(blob)
        if n < PREFIX_LEN:
            raise FormatMismatch(f".focrq truncated: {n} bytes < {PREFIX_LEN}-byte preamble")
        if bytes(blob[:6]) != MAGIC:
            raise FormatMismatch(".focrq bad magic")
        version, arch = struct.unpack_from("<IB", blob, 6)
        if version > FORMAT_VERSION:
            raise FormatMismatch(f".focrq format_version {version} is newer than this build "
                                 f"supports (max {FORMAT_VERSION})")
        prefix_sha = bytes(blob[11:43]).hex()
        (header_len,) = struct.unpack_from("<Q", blob, 43)
        header_end = PREFIX_LEN + header_len
        if header_end > n:
            raise FormatMismatch(f".focrq header ({header_len} bytes) overruns file ({n} bytes)")
        try:
            header = json.loads(bytes(blob[PREFIX_LEN:header_end]).decode("utf-8"))
        except (UnicodeDecodeError, json.JSONDecodeError) as e:
            raise FormatMismatch(f".focrq header JSON invalid: {e}") from e
        if not isinstance(header, dict) or not isinstance(header.get("tensors"), dict):
            raise FormatMismatch(".focrq header JSON invalid: missing tensors object")
        for key in ("model_id", "license_notice", "source_sha256"):
            if not isinstance(header.get(key, ""), str):
                raise FormatMismatch(f".focrq header JSON invalid: {key} must be a string")
        h_arch = header.get("arch_target", 0)
        if isinstance(h_arch, bool) or not isinstance(h_arch, int) or not 0 <= h_arch <= 255:
            raise FormatMismatch(".focrq header JSON invalid: arch_target must be a u8")
        model_id = resolve_model_id(header.get("model_id", ""))
        notice = header.get("license_notice", "")
        validate_license_notice(notice, model_id)
        h_sha = header.get("source_sha256", "")
        if h_sha:
            _validate_sha_hex(h_sha)
        directory = {name: _parse_record(name, r) for name, r in header["tensors"].items()}
        validate_directory(directory, n - header_end)
        return cls(blob, header_end, directory, h_arch if h_arch != 0 else arch,
                   h_sha or prefix_sha, notice, model_id, header)

    # -- directory -------------------------------------------------------------
    def __len__(self) -> int:
        return len(self.directory)

    def __contains__(self, name: str) -> bool:
        return name in self.directory

    def names(self):
        return sorted(self.directory)

    def record(self, name: str) -> TensorRecord:
        try:
            return self.directory[name]
        except KeyError:
            raise FormatMismatch(f"tensor {name!r} not found in weights directory") from None

    def census(self, expected_names) -> None:
        """Every expected name must be present (weights.rs:634-672)."""
        missing = [nm for nm in expected_names if nm not in self.directory]
        if missing:
            raise FormatMismatch(f"weights census: {len(missing)} expected tensors missing: "
                                 f"{missing[:8]}")

    def _payload(self, off: int, length: int) -> memoryview:
        s = self.payload_base + off
        return self._blob[s:s + length]

    # -- typed accessors -------------------------------------------------------
    def mat(self, name: str) -> np.ndarray:
        """A high-precision tensor widened exactly to f32, in its logical shape."""
        rec = self.record(name)
        data = self._payload(rec.byte_offset, rec.byte_len)
        if rec.dtype == "F32":
            out = np.frombuffer(data, dtype="<f4").astype(np.float32)
        elif rec.dtype == "F16":
            out = np.frombuffer(data, dtype="<f2").astype(np.float32)
        elif rec.dtype == "BF16":
            out = (np.frombuffer(data, dtype="<u2").astype(np.uint32) << 16).view(np.float32)
        else:
            raise FormatMismatch(f"tensor {name!r}: {rec.dtype} is quantized; use qint8()/qint4()")
        return out.reshape(rec.shape)

    def qint8(self, name: str) -> tuple[np.ndarray, np.ndarray]:
        """``QInt8PerChan`` -> (``[n, k]`` int8, ``[n]`` f32 scales)."""
        rec = self.record(name)
        if rec.dtype != "QInt8PerChan":
            raise FormatMismatch(f"tensor {name!r} is {rec.dtype}, not QInt8PerChan")
        if len(rec.shape) != 2:
            raise FormatMismatch(f"QInt8 tensor {name!r} has rank {len(rec.shape)}; expected 2")
        n, k = rec.shape
        q = np.frombuffer(self._payload(rec.byte_offset, rec.byte_len), dtype=np.int8)
        s = np.frombuffer(self._payload(rec.scales_offset, rec.scales_len), dtype="<f4")
        return q.reshape(n, k).copy(), s.astype(np.float32)

    def qint4(self, name: str) -> tuple[np.ndarray, np.ndarray, int]:
        """``QInt4PerGroup`` -> (``[n, k/2]`` packed u8, ``[n, k/g]`` f32 scales, g)."""
        rec = self.record(name)
        if rec.dtype != "QInt4PerGroup":
            raise FormatMismatch(f"tensor {name!r} is {rec.dtype}, not QInt4PerGroup")
        if len(rec.shape) != 2:
            raise FormatMismatch(f"QInt4 tensor {name!r} has rank {len(rec.shape)}; expected 2")
        n, k = rec.shape
        g = rec.group_size
        p = np.frombuffer(self._payload(rec.byte_offset, rec.byte_len), dtype=np.uint8)
        s = np.frombuffer(self._payload(rec.scales_offset, rec.scales_len), dtype="<f4")
        return p.reshape(n, k // 2).copy(), s.astype(np.float32).reshape(n, k // g), g

    def int8_rows(self, name: str) -> tuple[np.ndarray, np.ndarray]:
        """``quant_oc_loaded`` (decoder.rs:1777-1786): a stored ``QInt8PerChan``
        verbatim, else the high-precision matrix quantised per row."""
        if self.record(name).dtype == "QInt8PerChan":
            return self.qint8(name)
        return quantize_int8_f32(self.mat(name))


# -- writer ---------------------------------------------------------------------
class Writer:
    """Deterministic ``.focrq`` writer: sorted directory, canonical JSON header
    (sorted keys, no whitespace), 64-byte aligned ranges with zero padding,
    data before scales for each tensor in name order (src/quant/focrq.rs
    ``FocrqBuilder`` semantics, format document "Writer Determinism")."""

    def __init__(self, arch_target: int = 0, source_sha256: bytes = bytes(32),
                 license_notice: str = MODEL_LICENSE_NOTICE, model_id: str = "",
                 model_config: dict | None = None, packing_manifest: dict | None = None,
                 provenance: dict | None = None):
        if len(source_sha256) != 32:
            raise ValueError("source_sha256 must be 32 bytes")
        self.arch_target = arch_target
        self.source_sha256 = bytes(source_sha256)
        self.license_notice = license_notice
        self.model_id = model_id
        self.extra = {k: v for k, v in (("model_config", model_config),
                                        ("packing_manifest", packing_manifest),
                                        ("provenance", provenance)) if v is not None}
        self._t = {}

    def add_f32(self, name: str, a: np.ndarray) -> None:
        a = np.ascontiguousarray(a, dtype="<f4")
        self._t[name] = ("F32", a.shape, a.tobytes(), b"", 0, 0)

    def add_bf16(self, name: str, a: np.ndarray) -> None:
        """Stores the high 16 bits of each f32 (exact for bf16-representable
        values, which is what a bf16 checkpoint holds)."""
        a = np.ascontiguousarray(a, dtype=np.float32)
        hi = (a.view(np.uint32) >> 16).astype("<u2")
        self._t[name] = ("BF16", a.shape, hi.tobytes(), b"", 0, 0)

    def add_qint8(self, name: str, q: np.ndarray, scales: np.ndarray) -> None:
        q = np.ascontiguousarray(q, dtype=np.int8)
        s = np.ascontiguousarray(scales, dtype="<f4")
        if q.ndim != 2 or s.shape != (q.shape[0],):
            raise ValueError("add_qint8: q [n, k] with scales [n]")
        self._t[name] = ("QInt8PerChan", q.shape, q.tobytes(), s.tobytes(), 0, 0)

    def add_qint4(self, name: str, packed: np.ndarray, scales: np.ndarray, group: int,
                  tier: int = 0) -> None:
        p = np.ascontiguousarray(packed, dtype=np.uint8)
        s = np.ascontiguousarray(scales, dtype="<f4")
        n, k = p.shape[0], p.shape[1] * 2
        if group not in GROUP_SIZES or k % group or s.shape != (n, k // group):
            raise ValueError("add_qint4: packed [n, k/2], scales [n, k/group], group 16 or 32")
        self._t[name] = ("QInt4PerGroup", (n, k), p.tobytes(), s.tobytes(), group, tier)

    def to_bytes(self) -> bytes:
        payload = bytearray()
        tensors = {}

        def put(b: bytes) -> int:
            payload.extend(b"\0" * (-len(payload) % ALIGN))
            off = len(payload)
            payload.extend(b)
            return off

        for name in sorted(self._t):
            dtype, shape, data, scales, group, tier = self._t[name]
            rec = {"byte_len": len(data), "byte_offset": put(data), "dtype": dtype,
                   "shape": [int(d) for d in shape]}
            if dtype in ("QInt8PerChan", "QInt4PerGroup"):
                rec.update(scales_offset=put(scales), scales_len=len(scales), group_size=group,
                           tier=tier)
            tensors[name] = rec
        header = {"arch_target": self.arch_target, "format_version": FORMAT_VERSION,
                  "license_notice": self.license_notice,
                  "source_sha256": self.source_sha256.hex(), "tensors": tensors, **self.extra}
        if self.model_id:
            header["model_id"] = self.model_id
        hj = json.dumps(header, sort_keys=True, separators=(",", ":"),
                        ensure_ascii=False).encode("utf-8")
        return (MAGIC + struct.pack("<IB", FORMAT_VERSION, self.arch_target) +
                self.source_sha256 + struct.pack("<Q", len(hj)) + hj + bytes(payload))

    def write(self, path) -> None:
        with open(path, "wb") as f:
            f.write(self.to_bytes())


def sha256_bytes(b: bytes) -> bytes:
    return hashlib.sha256(b).digest()


# -- model mapping --------------------------------------------------------------
def layer_prefix(layer: int) -> str:
    return f"model.layers.{layer}.mlp"


def moe_tensor_names(layer: int, n_experts: int, shared: bool = True) -> list[str]:
    """The census of one MoE layer (decoder.rs:2057-2092)."""
    p = layer_prefix(layer)
    names = [f"{p}.gate.weight"]
    for e in range(n_experts):
        names += [f"{p}.experts.{e}.{r}_proj.weight" for r in ("gate", "up", "down")]
    if shared:
        names += [f"{p}.shared_experts.{r}_proj.weight" for r in ("gate", "up", "down")]
    return names


def moe_layer_weights(w: Weights, layer: int, topk: int = 6, expert_begin: int = 0,
                      expert_count: int | None = None) -> MoeWeightsHost:
    """One layer's MoE weights as :class:`MoeWeightsHost` for ``focr_moe_create``.

    The router ``[E, hidden]`` is read high precision; ``E`` comes from its
    shape.  Experts ``[expert_begin, expert_begin + expert_count)`` are loaded
    (an expert-parallel rank passes its own range).  All experts must share one
    storage kind: int8 (``QInt8PerChan`` or high precision, quantised per row)
    or ``QInt4PerGroup`` with a single group size.  The shared expert is
    optional; when present it is int8.
    """
    p = layer_prefix(layer)
    router = w.mat(f"{p}.gate.weight")
    if router.ndim != 2:
        raise FormatMismatch(f"{p}.gate.weight must be [n_experts, hidden]")
    n_experts, hidden = router.shape
    if expert_count is None:
        expert_count = n_experts - expert_begin
    if not (0 <= expert_begin and expert_count > 0 and expert_begin + expert_count <= n_experts):
        raise ValueError(f"expert range [{expert_begin}, {expert_begin + expert_count}) outside "
                         f"[0, {n_experts})")
    ids = range(expert_begin, expert_begin + expert_count)
    names = {r: [f"{p}.experts.{e}.{r}_proj.weight" for e in ids] for r in ("gate", "up", "down")}
    w.census([nm for v in names.values() for nm in v])
    kinds = {w.record(nm).dtype == "QInt4PerGroup" for v in names.values() for nm in v}
    if len(kinds) != 1:
        raise FormatMismatch(f"layer {layer}: experts mix QInt4PerGroup with int8 storage")
    int4 = kinds.pop()
    gate0 = w.record(names["gate"][0]).shape
    inter = gate0[0]
    want = {"gate": (inter, hidden), "up": (inter, hidden), "down": (hidden, inter)}
    for r, v in names.items():
        for nm in v:
            if tuple(w.record(nm).shape) != want[r]:
                raise FormatMismatch(f"tensor {nm!r}: shape {list(w.record(nm).shape)} != "
                                     f"{list(want[r])}")
    sh = [f"{p}.shared_experts.{r}_proj.weight" for r in ("gate", "up", "down")]
    has_shared = all(nm in w for nm in sh)
    if any(nm in w for nm in sh) and not has_shared:
        raise FormatMismatch(f"layer {layer}: incomplete shared expert")
    shared_inter = w.record(sh[0]).shape[0] if has_shared else 0

    group = 0
    out = MoeWeightsHost(hidden, inter, n_experts, topk, shared_inter, expert_begin,
                         expert_count, 0)
    out.router = np.ascontiguousarray(router, dtype=np.float32)
    for r, v in names.items():
        if int4:
            parts = [w.qint4(nm) for nm in v]
            gs = {g for _, _, g in parts}
            if len(gs) != 1 or (group and gs != {group}):
                raise FormatMismatch(f"layer {layer}: experts use more than one int4 group size")
            group = gs.pop()
            out.arrays[r + "_p"] = np.ascontiguousarray(np.stack([a for a, _, _ in parts]))
            out.arrays[r + "_gs"] = np.ascontiguousarray(np.stack([s for _, s, _ in parts]))
        else:
            parts = [w.int8_rows(nm) for nm in v]
            out.arrays[r + "_w"] = np.ascontiguousarray(np.stack([q for q, _ in parts]))
            out.arrays[r + "_s"] = np.ascontiguousarray(np.stack([s for _, s in parts]))
    out.group = group
    if has_shared:
        want_sh = {0: (shared_inter, hidden), 1: (shared_inter, hidden), 2: (hidden, shared_inter)}
        for i, (r, nm) in enumerate(zip(("sh_gate", "sh_up", "sh_down"), sh)):
            if tuple(w.record(nm).shape) != want_sh[i]:
                raise FormatMismatch(f"tensor {nm!r}: shape {list(w.record(nm).shape)} != "
                                     f"{list(want_sh[i])}")
            q, s = w.int8_rows(nm)
            out.arrays[r + "_w"] = q
            out.arrays[r + "_s"] = s
    return out


def lm_head_weights(w: Weights, row_begin: int = 0, rows: int | None = None,
                    name: str = "lm_head.weight") -> tuple[np.ndarray, np.ndarray]:
    """Rows ``[row_begin, row_begin + rows)`` of the int8 head (decoder.rs:2106):
    the vocab shard one rank owns."""
    q, s = w.int8_rows(name)
    if rows is None:
        rows = q.shape[0] - row_begin
    if not (0 <= row_begin and rows > 0 and row_begin + rows <= q.shape[0]):
        raise ValueError("lm-head row range outside the head")
    return (np.ascontiguousarray(q[row_begin:row_begin + rows]),
            np.ascontiguousarray(s[row_begin:row_begin + rows]))


def write_moe_layer(wr: Writer, layer: int, W: MoeWeightsHost) -> None:
    """Store a :class:`MoeWeightsHost` under the canonical names (the inverse
    of :func:`moe_layer_weights`; the router as F32)."""
    p = layer_prefix(layer)
    wr.add_f32(f"{p}.gate.weight", W.router)
    for i, e in enumerate(range(W.expert_begin, W.expert_begin + W.expert_count)):
        for r in ("gate", "up", "down"):
            nm = f"{p}.experts.{e}.{r}_proj.weight"
            if W.group:
                wr.add_qint4(nm, W.arrays[r + "_p"][i], W.arrays[r + "_gs"][i], W.group)
            else:
                wr.add_qint8(nm, W.arrays[r + "_w"][i], W.arrays[r + "_s"][i])
    if W.shared_inter:
        for r in ("gate", "up", "down"):
            wr.add_qint8(f"{p}.shared_experts.{r}_proj.weight", W.arrays["sh_" + r + "_w"],
                         W.arrays["sh_" + r + "_s"])


def decoder_tensor_names(n_layers: int, n_experts: int, first_dense: int = 1,
                         shared: bool = True) -> list[str]:
    """The census of the int8 decoder (DecoderWeightCacheI8::build,
    decoder.rs:2018-2117)."""
    names = ["model.embed_tokens.weight", "model.norm.weight", "lm_head.weight"]
    for l in range(n_layers):
        p = f"model.layers.{l}"
        names += [f"{p}.input_layernorm.weight", f"{p}.post_attention_layernorm.weight"]
        names += [f"{p}.self_attn.{r}_proj.weight" for r in ("q", "k", "v", "o")]
        if l < first_dense:
            names += [f"{p}.mlp.{r}_proj.weight" for r in ("gate", "up", "down")]
        else:
            names += moe_tensor_names(l, n_experts, shared)
    return names


def decoder_weights(w: Weights, n_layers: int | None = None, heads: int | None = None,
                    topk: int = 6):
    """The whole int8 decoder as a ``DecoderWeightsHost`` for ``DecoderI8``:
    per layer the two RMSNorm weights (high precision), the q/k/v/o
    projections and the dense MLP through ``quant_oc_loaded``, MoE layers
    through :func:`moe_layer_weights`; the final norm, the lm-head (int8) and
    the token embeddings (widened to f32).  A layer is MoE when its router
    ``mlp.gate.weight`` is present, dense otherwise; ``n_layers`` defaults to
    the number of ``model.layers.{l}`` prefixes in the directory (a smaller
    value loads that prefix of the layers).  ``heads`` defaults to the header's
    ``model_config.num_attention_heads`` (10 when absent); an explicit value
    that disagrees with it is a mismatch."""
    from .decoder import DecoderWeightsHost, LayerWeightsHost

    ls = {int(nm.split(".")[2]) for nm in w.directory if nm.startswith("model.layers.")}
    file_layers = max(ls) + 1 if ls else 0
    if n_layers is None:
        n_layers = file_layers
    cfg = w.header.get("model_config")
    cfg = cfg if isinstance(cfg, dict) else {}
    if heads is None:
        heads = int(cfg.get("num_attention_heads", 10))
    elif "num_attention_heads" in cfg and cfg["num_attention_heads"] != heads:
        raise FormatMismatch(f"model_config.num_attention_heads = {cfg['num_attention_heads']} "
                             f"but {heads} heads were asked for")
    if n_layers == 0:
        raise FormatMismatch("no decoder layers in the weights directory")
    embed = w.mat("model.embed_tokens.weight")
    if embed.ndim != 2:
        raise FormatMismatch("model.embed_tokens.weight must be [vocab, hidden]")
    vocab, hidden = embed.shape
    layers = []
    for l in range(n_layers):
        p = f"model.layers.{l}"
        L = LayerWeightsHost(input_ln=w.mat(f"{p}.input_layernorm.weight").reshape(-1),
                             post_ln=w.mat(f"{p}.post_attention_layernorm.weight").reshape(-1))
        if L.input_ln.shape != (hidden,) or L.post_ln.shape != (hidden,):
            raise FormatMismatch(f"{p}: layer norms must have {hidden} elements")
        for r in ("q", "k", "v", "o"):
            L.proj[r + "_w"], L.proj[r + "_s"] = w.int8_rows(f"{p}.self_attn.{r}_proj.weight")
        D = heads * 128
        want = {"q": (D, hidden), "k": (D, hidden), "v": (D, hidden), "o": (hidden, D)}
        for r, shp in want.items():
            if L.proj[r + "_w"].shape != shp:
                raise FormatMismatch(f"{p}.self_attn.{r}_proj.weight: shape "
                                     f"{list(L.proj[r + '_w'].shape)} != {list(shp)}")
        if f"{p}.mlp.gate.weight" in w:
            L.moe = moe_layer_weights(w, l, topk=topk)
            if L.moe.hidden != hidden:
                raise FormatMismatch(f"{p}: router hidden {L.moe.hidden} != {hidden}")
        else:
            L.dense = {}
            for r in ("gate", "up", "down"):
                L.dense[r + "_w"], L.dense[r + "_s"] = w.int8_rows(f"{p}.mlp.{r}_proj.weight")
            I = L.dense["gate_w"].shape[0]
            for r, shp in (("gate", (I, hidden)), ("up", (I, hidden)), ("down", (hidden, I))):
                if L.dense[r + "_w"].shape != shp:
                    raise FormatMismatch(f"{p}.mlp.{r}_proj.weight: shape "
                                         f"{list(L.dense[r + '_w'].shape)} != {list(shp)}")
        layers.append(L)
    # format document "Frozen model_config": a mismatch with the tensors is
    # FormatMismatch, not a warning.  The layer count is the file's, not the
    # (possibly smaller) number of layers asked for.
    for key, have in (("hidden_size", hidden), ("num_attention_heads", heads),
                      ("num_hidden_layers", file_layers), ("vocab_size", vocab)):
        if key in cfg and cfg[key] != have:
            raise FormatMismatch(f"model_config.{key} = {cfg[key]} but the tensors give {have}")
    lm_w, lm_s = w.int8_rows("lm_head.weight")
    if lm_w.shape != (vocab, hidden):
        raise FormatMismatch(f"lm_head.weight: shape {list(lm_w.shape)} != {[vocab, hidden]}")
    final = w.mat("model.norm.weight").reshape(-1)
    return DecoderWeightsHost(hidden=hidden, heads=heads, vocab=vocab, layers=layers,
                              final_norm=np.ascontiguousarray(final, dtype=np.float32),
                              lm_w=lm_w, lm_s=lm_s,
                              embed=np.ascontiguousarray(embed, dtype=np.float32))


def write_decoder(wr: Writer, W) -> None:
    """Store a ``DecoderWeightsHost`` under the canonical names (norms,
    router and embeddings as F32; projections and experts as stored)."""
    wr.add_f32("model.embed_tokens.weight", W.embed)
    wr.add_f32("model.norm.weight", W.final_norm)
    wr.add_qint8("lm_head.weight", W.lm_w, W.lm_s)
    for l, L in enumerate(W.layers):
        p = f"model.layers.{l}"
        wr.add_f32(f"{p}.input_layernorm.weight", L.input_ln)
        wr.add_f32(f"{p}.post_attention_layernorm.weight", L.post_ln)
        for r in ("q", "k", "v", "o"):
            wr.add_qint8(f"{p}.self_attn.{r}_proj.weight", L.proj[r + "_w"], L.proj[r + "_s"])
        if L.moe is not None:
            write_moe_layer(wr, l, L.moe)
        else:
            for r in ("gate", "up", "down"):
                wr.add_qint8(f"{p}.mlp.{r}_proj.weight", L.dense[r + "_w"], L.dense[r + "_s"])
