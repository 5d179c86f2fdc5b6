"""safetensors reading (zero-copy) and writing, and the native block-scaled weight pairs of
DeepSeek-V4-style checkpoints.

Container: an 8-byte little-endian header length, a JSON header (tensor name -> dtype, shape and
[begin, end) byte offsets into the data section; an optional ``__metadata__`` string map), then
the data section. Payloads are exposed as read-only numpy views of one file mapping.

Native pairs: a tensor ``<stem>.weight`` of dtype ``I8`` or ``F8_E4M3`` is paired with the
``F8_E8M0`` tensor ``<stem>.scale``:

* ``I8 [out, K / 2]``: two fp4 e2m1 codes per byte (column c in byte c / 2, the high nibble for
  odd c) with one e8m0 exponent per 32 columns, scale ``[out, K / 32]``;
* ``F8_E4M3 [out, K]``: fp8 e4m3 with one e8m0 exponent per 128 x 128 block, scale
  ``[out / 128, K / 128]``.

A weight whose scale is missing, not rank-two E8M0 or not of the exact shape, a weight name that
does not end in ``.weight``, and an E8M0 tensor that no weight claims are errors. The pairs load
as mixed-table weights (kinds FP4 and FP8) with the exponents as exact fp32 scales (2^(e - 127)).
DeepSeek-V3 / R1 checkpoints pair an ``F8_E4M3`` ``<stem>.weight`` with an ``F32``
``<stem>.weight_scale_inv`` [ceil(out / 128), K / 128] of per-block multipliers instead; those load
as kind FP8 too. ``act_quant_e8m0`` and ``fp8_block_matvec`` state the source checkpoint's own fp8 linear (e4m3
activations with a power-of-two scale per 128 columns) as a host reference.

Parity: crates/hawking-core/src/gravity_deepseek_v4.rs:114-160 (NativeScalePairKind /
NativeScalePairGeometry) and :2036-2125 (validate_native_scale_pairs).
"""
from __future__ import annotations

import json
import mmap
import struct
from dataclasses import dataclass
from typing import Dict, List, Mapping, Optional, Tuple

import numpy as np
import torch

# element sizes of the dtypes this reader hands out as raw bytes
DTYPE_BYTES = {"BOOL": 1, "U8": 1, "I8": 1, "F8_E4M3": 1, "F8_E5M2": 1, "F8_E8M0": 1, "I16": 2, "U16": 2,
               "F16": 2, "BF16": 2, "I32": 4, "U32": 4, "F32": 4, "I64": 8, "U64": 8, "F64": 8}
FP4_BLOCK = 32    # logical columns per e8m0 exponent of an fp4 weight
FP8_BLOCK = 128   # rows and columns of one e8m0 block of an fp8 weight


class SafetensorsError(ValueError):
    pass


@dataclass
class StTensor:
    name: str
    dtype: str
    shape: Tuple[int, ...]
    begin: int           # byte offsets into the data section
    end: int

    @property
    def nbytes(self) -> int:
        return self.end - self.begin


class SafeTensors:
    """A safetensors file mapped read-only."""

    def __init__(self, path: str):
        self.path = path
        with open(path, "rb") as f:
            self._mm = mmap.mmap(f.fileno(), 0, access=mmap.ACCESS_READ)
        if len(self._mm) < 8:
            raise SafetensorsError(f"{path}: too short for a safetensors header")
        (n,) = struct.unpack_from("<Q", self._mm, 0)
        if 8 + n > len(self._mm):
            raise SafetensorsError(f"{path}: header length {n} past the end of the file")
        try:
            header = json.loads(bytes(self._mm[8:8 + n]).decode("utf-8"))
        except (UnicodeDecodeError, json.JSONDecodeError) as e:
            raise SafetensorsError(f"{path}: header is not JSON ({e})") from e
        self.metadata: Dict[str, str] = header.pop("__metadata__", {}) or {}
        self._data0 = 8 + n
        data_len = len(self._mm) - self._data0
        self.tensors: Dict[str, StTensor] = {}
        for name, h in header.items():
            dtype, shape, (b, e) = h["dtype"], tuple(int(d) for d in h["shape"]), h["data_offsets"]
            if dtype not in DTYPE_BYTES:
                raise SafetensorsError(f"{name}: unsupported dtype {dtype}")
            want = int(np.prod(shape, dtype=np.int64)) * DTYPE_BYTES[dtype] if shape else DTYPE_BYTES[dtype]
            if not (0 <= b <= e <= data_len) or e - b != want:
                raise SafetensorsError(f"{name}: offsets [{b}, {e}) do not hold {dtype}{list(shape)}")
            self.tensors[name] = StTensor(name, dtype, shape, int(b), int(e))

    def names(self) -> List[str]:
        return sorted(self.tensors)

    def raw(self, name: str) -> np.ndarray:
        """The tensor's bytes as a read-only uint8 view [nbytes]."""
        t = self.tensors[name]
        return np.frombuffer(self._mm, dtype=np.uint8, count=t.nbytes, offset=self._data0 + t.begin)

    def close(self):
        self._mm.close()


def write_safetensors(path: str, tensors: Mapping[str, Tuple[str, Tuple[int, ...], bytes]],
                      metadata: Optional[Mapping[str, str]] = None) -> str:
    """Write ``name -> (dtype, shape, payload bytes)`` in name order (8-byte aligned header)."""
    header: Dict[str, object] = {}
    off = 0
    blobs = []
    for name in sorted(tensors):
        dtype, shape, data = tensors[name]
        data = bytes(data)
        header[name] = {"dtype": dtype, "shape": list(shape), "data_offsets": [off, off + len(data)]}
        blobs.append(data)
        off += len(data)
    if metadata:
        header["__metadata__"] = dict(metadata)
    hb = json.dumps(header, separators=(",", ":")).encode("utf-8")
    hb += b" " * (-len(hb) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(hb)))
        f.write(hb)
        for b in blobs:
            f.write(b)
    return path


@dataclass
class NativePair:
    kind: str            # "native.fp4_e2m1fn_x2_e8m0", "native.fp8_e4m3fn_e8m0" or "native.fp8_e4m3fn_f32" (V3 weight_scale_inv)
    weight: str
    scale: str
    out_rows: int
    packed_k: int
    logical_k: int
    scale_rows: int
    scale_cols: int


def native_scale_pairs(st: SafeTensors) -> Dict[str, NativePair]:
    """Pair every native fp4 / fp8 weight with its e8m0 scale tensor, checking the geometry."""
    pairs: Dict[str, NativePair] = {}
    claimed = set()
    for name in st.names():
        w = st.tensors[name]
        if w.dtype == "F8_E4M3" and name.endswith(".weight") and name + "_scale_inv" in st.tensors:
            # DeepSeek-V3 / R1 convention: fp32 multipliers per 128 x 128 block (edge blocks partial)
            s = st.tensors[name + "_scale_inv"]
            if s.dtype != "F32" or len(w.shape) != 2 or len(s.shape) != 2:
                raise SafetensorsError(f"{name}: weight_scale_inv must be a rank-two F32 tensor")
            out_rows, k = w.shape
            if k % FP8_BLOCK:
                raise SafetensorsError(f"{name}: fp8 K {k} is not a multiple of {FP8_BLOCK}")
            want = (-(-out_rows // FP8_BLOCK), k // FP8_BLOCK)
            if tuple(s.shape) != want:
                raise SafetensorsError(f"{name}: weight_scale_inv shape {list(s.shape)}, expected {list(want)}")
            pairs[name] = NativePair("native.fp8_e4m3fn_f32", name, s.name, out_rows, k, k, *want)
            continue
        if w.dtype == "I8":
            kind = "native.fp4_e2m1fn_x2_e8m0"
        elif w.dtype == "F8_E4M3":
            kind = "native.fp8_e4m3fn_e8m0"
        else:
            continue
        if not name.endswith(".weight"):
            raise SafetensorsError(f"{name}: a native {kind} weight must be named <stem>.weight")
        sname = name[: -len(".weight")] + ".scale"
        s = st.tensors.get(sname)
        if s is None:
            raise SafetensorsError(f"{name}: no matching E8M0 scale tensor {sname}")
        if s.dtype != "F8_E8M0" or len(w.shape) != 2 or len(s.shape) != 2:
            raise SafetensorsError(f"{name}: the weight / scale pair is not rank-two with E8M0 scales")
        out_rows, packed_k = w.shape
        if kind == "native.fp4_e2m1fn_x2_e8m0":
            logical_k = 2 * packed_k
            if logical_k % FP4_BLOCK:
                raise SafetensorsError(f"{name}: fp4 logical K {logical_k} is not a multiple of {FP4_BLOCK}")
            srows, scols = out_rows, logical_k // FP4_BLOCK
        else:
            logical_k = packed_k
            if out_rows % FP8_BLOCK or packed_k % FP8_BLOCK:
                raise SafetensorsError(f"{name}: fp8 dimensions must be multiples of {FP8_BLOCK}")
            srows, scols = out_rows // FP8_BLOCK, packed_k // FP8_BLOCK
        if tuple(s.shape) != (srows, scols):
            raise SafetensorsError(f"{name}: scale shape {list(s.shape)}, expected {[srows, scols]}")
        pairs[name] = NativePair(kind, name, sname, out_rows, packed_k, logical_k, srows, scols)
        claimed.add(sname)
    for name in st.names():
        if st.tensors[name].dtype == "F8_E8M0" and name not in claimed:
            raise SafetensorsError(f"{name}: E8M0 scale tensor without a native weight")
    return pairs


def _e8m0_scales(raw: np.ndarray) -> torch.Tensor:
    e = torch.from_numpy(raw.astype(np.int32))
    if bool((e == 255).any()):
        raise SafetensorsError("e8m0 exponent 255 (NaN) in a scale tensor")
    return torch.exp2((e - 127).float())


def load_native_pair(st: SafeTensors, pair: NativePair, device):
    """The pair as a mixed-table weight: kind FP4 (codes kept, fp32 scale per 32 columns) or kind
    FP8 (codes kept, fp32 scale per 128 columns of each row, from the 128 x 128 blocks)."""
    from ..ops.mixed import FP8, MixedWeight
    codes = torch.from_numpy(np.array(st.raw(pair.weight))).view(pair.out_rows, pair.packed_k)
    if pair.kind == "native.fp4_e2m1fn_x2_e8m0":
        e8 = torch.from_numpy(np.array(st.raw(pair.scale))).view(pair.scale_rows, pair.scale_cols)
        return MixedWeight.from_e2m1_e8m0(codes, e8, pair.out_rows, pair.logical_k, device)
    if pair.kind == "native.fp8_e4m3fn_f32":
        sc = torch.from_numpy(np.array(st.raw(pair.scale)).view(np.float32)).view(pair.scale_rows, pair.scale_cols)
    else:
        sc = _e8m0_scales(st.raw(pair.scale)).view(pair.scale_rows, pair.scale_cols)
    rows = sc.repeat_interleave(FP8_BLOCK, 0)[: pair.out_rows].contiguous()  # [out, K / 128]
    return MixedWeight(FP8, 8, FP8_BLOCK, pair.out_rows, pair.logical_k, codes.to(device).contiguous(),
                       rows.to(device))


# ---- block-scaled activation quantisation of the native fp8 linears --------------------------
ACT_BLOCK = 128          # activation columns per e8m0 scale
E4M3_MAX = 448.0
ACT_AMAX_FLOOR = 1.0e-4  # a block's absolute maximum is raised to this before its scale is taken


def act_quant_e8m0(x: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """Quantise activation rows [..., K] (K % 128 == 0) the way the native fp8 linears expect:
    per block of 128 columns the scale is the power of two at or above max(amax, 1e-4) * (1 / 448)
    (the fp32 product; the power from its exponent bits, one up when the mantissa is nonzero),
    stored as its e8m0 byte, and each element is x / scale clamped to +-448 and rounded to fp8
    e4m3 (nearest, ties to even). Returns (e4m3 bytes [..., K] uint8, e8m0 bytes [..., K / 128]).

    Parity: crates/hawking-core/src/gravity_deepseek_v4_act_quant.rs:221-300
    (rounded_ue8m0_scale_byte, act_quant_bf16_ue8m0)."""
    xf = x.float()
    K = xf.shape[-1]
    if K % ACT_BLOCK:
        raise ValueError("act_quant_e8m0: K must be a multiple of 128")
    if not bool(torch.isfinite(xf).all()):
        raise ValueError("act_quant_e8m0: non-finite activation")
    blocks = xf.reshape(*xf.shape[:-1], K // ACT_BLOCK, ACT_BLOCK)
    amax = blocks.abs().amax(-1).clamp_min(ACT_AMAX_FLOOR)
    scaled = amax * torch.tensor(1.0 / E4M3_MAX, dtype=torch.float32)   # the fp32 product
    bits = scaled.contiguous().view(torch.int32)
    exp = ((bits >> 23) & 0xFF) - 127 + ((bits & 0x7FFFFF) != 0).to(torch.int32)
    e8 = exp + 127
    if bool(((e8 < 0) | (e8 > 254)).any()):
        raise ValueError("act_quant_e8m0: scale outside the finite e8m0 range")
    scale = torch.exp2(exp.float())
    q = (blocks / scale.unsqueeze(-1)).clamp(-E4M3_MAX, E4M3_MAX).to(torch.float8_e4m3fn)
    return q.view(torch.uint8).reshape(xf.shape), e8.to(torch.uint8)


def fp8_block_matvec(w_e4m3: torch.Tensor, w_e8m0: torch.Tensor, a_e4m3: torch.Tensor, a_e8m0: torch.Tensor
                     ) -> torch.Tensor:
    """y [rows] of a native fp8 weight ([rows, K] e4m3 bytes, e8m0 [rows / 128, K / 128]) times one
    quantised activation row (e4m3 bytes [K], e8m0 [K / 128]): per 128-column block the fp32 dot
    of the decoded codes times the product of the two scales, summed over the blocks in order."""
    rows, K = w_e4m3.shape
    w = w_e4m3.view(torch.float8_e4m3fn).float().view(rows, K // ACT_BLOCK, ACT_BLOCK)
    a = a_e4m3.view(torch.float8_e4m3fn).float().view(K // ACT_BLOCK, ACT_BLOCK)
    ws = torch.exp2(w_e8m0.float() - 127).repeat_interleave(FP8_BLOCK, 0)[:rows]   # [rows, K / 128]
    sa = torch.exp2(a_e8m0.float() - 127)                                         # [K / 128]
    dots = (w * a.unsqueeze(0)).sum(-1)                                           # [rows, K / 128]
    return (dots * (ws * sa.unsqueeze(0))).sum(-1)
