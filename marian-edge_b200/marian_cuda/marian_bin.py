"""Marian binary format v1 (``*.intgemm.alphas.bin``): writer and strict reader.

The rules follow ``crates/marian-cpu/src/legacy_q8.rs`` of marian-edge:

* header: u64 version (=1), u64 tensor count, then per tensor u64 name length
  (including the NUL), u64 type, u64 rank, u64 payload length
  (legacy_q8.rs:179-226);
* names (NUL-terminated UTF-8), then shapes as i32 (legacy_q8.rs:228-285);
* u64 padding length followed by that many zero bytes so tensor data starts on
  a 256-byte boundary (legacy_q8.rs:287-299);
* payloads: raw int8 records unpadded; float32 and intgemm8 records padded with
  zeros to 256 bytes (legacy_q8.rs:301-330).  An intgemm8 record holds the int8
  values followed by its f32 ``quant_mult`` (legacy_q8.rs:378-410).

Dense intgemm tensors declare a ``[input, output]`` header shape while their
bytes are canonical ``[output, input]``; ``*_Wemb`` tensors are
``[vocabulary, dimension]`` in both (legacy_q8.rs:80-87).

The CUDA library parses the same bytes independently in C++
(``csrc/model_loader.cpp``); tests feed both parsers the files written here.
"""
from __future__ import annotations

import struct
from dataclasses import dataclass
from typing import Iterable

import numpy as np

TYPE_INT8 = 0x0101
TYPE_FLOAT32 = 0x0404
TYPE_INTGEMM8 = 0x4101
DATA_ALIGNMENT = 256
MAXIMUM_FILE_BYTES = 128 * 1024 * 1024
MAXIMUM_TENSORS = 4096
MAXIMUM_NAME_BYTES = 16 * 1024
MAXIMUM_RANK = 8


class MarianFormatError(ValueError):
    pass


@dataclass
class Tensor:
    name: str
    tensor_type: int
    shape: tuple
    # float32 -> np.float32 array; int8 -> np.int8 array;
    # intgemm8 -> (np.int8 array, float quant_mult)
    data: object

    def payload(self) -> bytes:
        if self.tensor_type == TYPE_INT8:
            return np.asarray(self.data, dtype=np.int8).tobytes()
        if self.tensor_type == TYPE_FLOAT32:
            raw = np.asarray(self.data, dtype="<f4").tobytes()
        elif self.tensor_type == TYPE_INTGEMM8:
            values, quant_mult = self.data
            raw = np.asarray(values, dtype=np.int8).tobytes() + struct.pack("<f", float(quant_mult))
        else:
            raise MarianFormatError(f"unsupported tensor type 0x{self.tensor_type:04x}")
        padded = -(-len(raw) // DATA_ALIGNMENT) * DATA_ALIGNMENT
        return raw + b"\0" * (padded - len(raw))


def f32(name: str, values, shape=None) -> Tensor:
    arr = np.asarray(values, dtype=np.float32)
    return Tensor(name, TYPE_FLOAT32, tuple(shape if shape is not None else arr.shape), arr.ravel())


def q8(name: str, values, quant_mult: float, shape) -> Tensor:
    arr = np.asarray(values, dtype=np.int8)
    return Tensor(name, TYPE_INTGEMM8, tuple(shape), (arr.ravel(), float(quant_mult)))


def raw_int8(name: str, data: bytes) -> Tensor:
    arr = np.frombuffer(data, dtype=np.int8)
    return Tensor(name, TYPE_INT8, (len(arr),), arr)


def write(tensors: Iterable[Tensor]) -> bytes:
    tensors = list(tensors)
    out = bytearray()
    out += struct.pack("<QQ", 1, len(tensors))
    payloads = [t.payload() for t in tensors]
    for t, p in zip(tensors, payloads):
        name = t.name.encode("utf-8")
        out += struct.pack("<QQQQ", len(name) + 1, t.tensor_type, len(t.shape), len(p))
    for t in tensors:
        out += t.name.encode("utf-8") + b"\0"
    for t in tensors:
        out += struct.pack(f"<{len(t.shape)}i", *t.shape)
    pad = (-(len(out) + 8)) % DATA_ALIGNMENT
    out += struct.pack("<Q", pad) + b"\0" * pad
    for p in payloads:
        out += p
    return bytes(out)


def _logical_bytes(tensor_type: int, elements: int) -> int:
    if tensor_type == TYPE_INT8:
        return elements
    if tensor_type == TYPE_FLOAT32:
        return elements * 4
    return elements + 4


def parse(data: bytes) -> dict:
    """Strict parse; returns {name: Tensor} in file order (legacy_q8.rs:179-422)."""
    if len(data) > MAXIMUM_FILE_BYTES:
        raise MarianFormatError("model exceeds the maximum file size")
    pos = 0

    def take(n):
        nonlocal pos
        if n < 0 or pos + n > len(data):
            raise MarianFormatError(f"truncated: need {n} bytes at {pos}")
        chunk = data[pos:pos + n]
        pos += n
        return chunk

    version, count = struct.unpack("<QQ", take(16))
    if version != 1:
        raise MarianFormatError(f"unsupported version {version}; expected 1")
    if not 1 <= count <= MAXIMUM_TENSORS:
        raise MarianFormatError(f"tensor count {count} is outside 1..={MAXIMUM_TENSORS}")
    headers = []
    for i in range(count):
        name_len, ttype, rank, dlen = struct.unpack("<QQQQ", take(32))
        if ttype not in (TYPE_INT8, TYPE_FLOAT32, TYPE_INTGEMM8):
            raise MarianFormatError(f"unsupported tensor type 0x{ttype:04x}")
        if not 2 <= name_len <= MAXIMUM_NAME_BYTES:
            raise MarianFormatError(f"header {i} name length {name_len} out of range")
        if not 1 <= rank <= MAXIMUM_RANK:
            raise MarianFormatError(f"header {i} rank {rank} out of range")
        if dlen == 0 or dlen > MAXIMUM_FILE_BYTES:
            raise MarianFormatError(f"header {i} has invalid data length {dlen}")
        headers.append((name_len, ttype, rank, dlen))
    names = []
    for i, (name_len, *_rest) in enumerate(headers):
        raw = take(name_len)
        if raw[-1] != 0 or 0 in raw[:-1]:
            raise MarianFormatError(f"tensor {i} name is not one NUL-terminated string")
        name = raw[:-1].decode("utf-8")
        if name in names:
            raise MarianFormatError(f"duplicate tensor name {name}")
        names.append(name)
    shapes = []
    for i, (_, _, rank, _) in enumerate(headers):
        dims = struct.unpack(f"<{rank}i", take(4 * rank))
        if any(d <= 0 for d in dims):
            raise MarianFormatError(f"tensor {names[i]} has a non-positive shape dimension")
        shapes.append(tuple(dims))
    (pad,) = struct.unpack("<Q", take(8))
    if any(take(pad)):
        raise MarianFormatError("header alignment padding contains non-zero bytes")
    if pos % DATA_ALIGNMENT:
        raise MarianFormatError("tensor data is not 256-byte aligned")
    tensors = {}
    for i, (_, ttype, _, dlen) in enumerate(headers):
        name, shape = names[i], shapes[i]
        elements = int(np.prod(shape))
        payload = take(dlen)
        logical = _logical_bytes(ttype, elements)
        expected = logical if ttype == TYPE_INT8 else -(-logical // DATA_ALIGNMENT) * DATA_ALIGNMENT
        if dlen != expected:
            raise MarianFormatError(f"{name}: record length {dlen}, expected {expected}")
        if any(payload[logical:]):
            raise MarianFormatError(f"{name}: record padding contains non-zero bytes")
        if ttype == TYPE_INT8:
            value = np.frombuffer(payload[:elements], dtype=np.int8).copy()
        elif ttype == TYPE_FLOAT32:
            value = np.frombuffer(payload[:logical], dtype="<f4").copy()
            if not np.all(np.isfinite(value)):
                raise MarianFormatError(f"{name}: float32 payload is not finite")
        else:
            values = np.frombuffer(payload[:elements], dtype=np.int8).copy()
            if (values == -128).any():
                raise MarianFormatError(f"{name}: symmetric intgemm8 payload contains -128")
            (qm,) = struct.unpack("<f", payload[elements:elements + 4])
            if not np.isfinite(qm) or qm <= 0:
                raise MarianFormatError(f"{name}: intgemm8 quantization multiplier must be finite and positive")
            value = (values, np.float32(qm))
        tensors[name] = Tensor(name, ttype, shape, value)
    if pos != len(data):
        raise MarianFormatError(f"{len(data) - pos} trailing bytes remain after the final tensor")
    return tensors


def activation_scale(tensors: dict, weight_name: str) -> np.float32:
    """Static activation alpha for a Q8 weight (legacy_q8.rs:549-552, 646-674).

    A float32 scalar is used as is; an accidentally quantized intgemm8 scalar
    is normalised as ``q / quant_mult``.
    """
    t = tensors.get(weight_name + "_QuantMultA")
    if t is None:
        raise MarianFormatError(f"missing tensor {weight_name}_QuantMultA")
    if int(np.prod(t.shape)) != 1:
        raise MarianFormatError(f"{t.name}: activation scale must be scalar")
    if t.tensor_type == TYPE_FLOAT32:
        scale = np.float32(t.data[0])
    elif t.tensor_type == TYPE_INTGEMM8:
        values, qm = t.data
        scale = np.float32(np.float32(values[0]) / np.float32(qm))
    else:
        raise MarianFormatError(f"{t.name}: activation scale must be float32 or intgemm8")
    if not np.isfinite(scale) or scale <= 0:
        raise MarianFormatError(f"{t.name}: activation scale must be finite and positive")
    return scale
