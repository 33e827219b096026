"""GGUF F32 export and import of a model's parameters, in the reference's layout
(save_gguf / load_gguf, src/gguf.cpp:355-497, 582-735):

- header: magic "GGUF", version 3, tensor count, KV count (little-endian u32, u32, u64, u64);
- six string KVs (type 8): general.architecture "llm", general.name "llm-cpp",
  llm.vocab_size, llm.n_embd (from the first parameter's shape), llm.block_size (from the
  second's first dimension), llm.tensor_count; a string is a u64 length and its bytes;
- one info per parameter, in parameters() order: name "tensor_<i>", u32 dimension count,
  the u64 dimensions in the parameter's own order, u32 type (0 = F32), u64 offset of its
  data from the start of the data section, offsets aligned to 32 bytes;
- zero padding to a 32-byte boundary, then each tensor's fp32 data at its offset.

Reading accepts F32 tensors only and checks the tensor count and every shape against the
model. `write_gguf_quant` writes the reference's quantized export (save_gguf_quant,
src/gguf.cpp:499-581) for qtype 0 (F32), 8 (Q8_0: per 32 values an f32 scale
max|x| / 127 + 1e-8 and 32 int8) and 4 (Q4_0: scale max|x| / 7 + 1e-8 and 16 bytes of
nibbles, value + 8, even index in the low nibble), with the extra KV llm.quant_type; values
are rounded half away from zero as std::round does. Q4_K (qtype 12) is not written.
"""
import struct

import numpy as np

GGUF_MAGIC = 0x46554747
GGUF_VERSION = 3
GGUF_TYPE_STRING = 8
GGUF_F32 = 0
GGUF_ALIGN = 32


def _align(n):
    return (n + GGUF_ALIGN - 1) & ~(GGUF_ALIGN - 1)


def _string(s):
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


def write_gguf(path, arrays):
    """Writes fp32 arrays (parameters() order) as the reference's save_gguf does."""
    arrays = [np.ascontiguousarray(a, dtype=np.float32) for a in arrays]
    vocab = n_embd = block = 0
    if len(arrays) >= 2:
        if arrays[0].ndim >= 2:
            vocab, n_embd = arrays[0].shape[0], arrays[0].shape[1]
        if arrays[1].ndim >= 2:
            block = arrays[1].shape[0]
    kvs = [("general.architecture", "llm"), ("general.name", "llm-cpp"),
           ("llm.vocab_size", str(vocab)), ("llm.n_embd", str(n_embd)),
           ("llm.block_size", str(block)), ("llm.tensor_count", str(len(arrays)))]
    out = bytearray(struct.pack("<IIQQ", GGUF_MAGIC, GGUF_VERSION, len(arrays), len(kvs)))
    for k, v in kvs:
        out += _string(k) + struct.pack("<I", GGUF_TYPE_STRING) + _string(v)
    offsets, cur = [], 0
    for a in arrays:
        cur = _align(cur)
        offsets.append(cur)
        cur += a.nbytes
    for i, (a, off) in enumerate(zip(arrays, offsets)):
        out += _string(f"tensor_{i}") + struct.pack("<I", a.ndim)
        out += struct.pack(f"<{a.ndim}Q", *a.shape) + struct.pack("<IQ", GGUF_F32, off)
    out += bytes(_align(len(out)) - len(out))
    data_start = len(out)
    for a, off in zip(arrays, offsets):
        out += bytes(data_start + off - len(out))
        out += a.tobytes()
    with open(path, "wb") as f:
        f.write(out)


GGUF_Q4_0 = 2
GGUF_Q8_0 = 8
_QBLK = 32


def _round_away(v):
    """std::round of float32 values (half away from zero), exact in float64."""
    v64 = v.astype(np.float64)
    return (np.sign(v64) * np.floor(np.abs(v64) + 0.5)).astype(np.float32)


def _encode(a, qtype):
    x = np.ascontiguousarray(a, dtype=np.float32).ravel()
    if qtype == 0:
        return x.tobytes()
    x = np.concatenate([x, np.zeros((-x.size) % _QBLK, np.float32)]).reshape(-1, _QBLK)
    mx = np.abs(x).max(axis=1)
    top = np.float32(127.0 if qtype == 8 else 7.0)
    sc = (mx / top).astype(np.float32) + np.float32(1e-8)
    q = _round_away((x / sc[:, None]).astype(np.float32))
    if qtype == 8:
        body = np.clip(q, -127, 127).astype(np.int8).view(np.uint8)
    else:
        q = np.clip(q, -8, 7).astype(np.int32) + 8
        body = ((q[:, 1::2] << 4) | (q[:, 0::2] & 0xF)).astype(np.uint8)
    return np.concatenate([sc[:, None].view(np.uint8), body], axis=1).tobytes()


def write_gguf_quant(path, arrays, qtype):
    """The reference's save_gguf_quant for qtype 0 (F32), 8 (Q8_0) or 4 (Q4_0)."""
    dtype = {0: GGUF_F32, 8: GGUF_Q8_0, 4: GGUF_Q4_0}.get(qtype)
    if dtype is None:
        raise ValueError(f"gguf: quant type {qtype} is not written here (0, 8 and 4 are)")
    arrays = [np.asarray(a, dtype=np.float32) for a in arrays]
    vocab = arrays[0].shape[0] if arrays else 0
    n_embd = arrays[0].shape[1] if arrays else 0
    block = arrays[1].shape[0] if len(arrays) >= 2 else 0
    kvs = [("general.architecture", "llm"), ("general.name", "llm-cpp"),
           ("llm.vocab_size", str(vocab)), ("llm.n_embd", str(n_embd)),
           ("llm.block_size", str(block)), ("llm.tensor_count", str(len(arrays))),
           ("llm.quant_type", str(qtype))]
    out = bytearray(struct.pack("<IIQQ", GGUF_MAGIC, GGUF_VERSION, len(arrays), len(kvs)))
    for k, v in kvs:
        out += _string(k) + struct.pack("<I", GGUF_TYPE_STRING) + _string(v)
    blobs = [_encode(a, qtype) for a in arrays]
    offsets, cur = [], 0
    for b in blobs:
        cur = _align(cur)
        offsets.append(cur)
        cur += len(b)
    for i, (a, off) in enumerate(zip(arrays, offsets)):
        out += _string(f"tensor_{i}") + struct.pack("<I", a.ndim)
        out += struct.pack(f"<{a.ndim}Q", *a.shape) + struct.pack("<IQ", dtype, off)
    out += bytes(_align(len(out)) - len(out))
    data_start = len(out)
    for b, off in zip(blobs, offsets):
        out += bytes(data_start + off - len(out))
        out += b
    with open(path, "wb") as f:
        f.write(out)


def read_gguf(path, shapes=None):
    """Reads an F32 GGUF written in the reference's layout; returns (arrays, kvs). With
    `shapes`, the tensor count and every shape must match (as load_gguf checks)."""
    with open(path, "rb") as f:
        buf = f.read()
    pos = 0

    def take(fmt):
        nonlocal pos
        v = struct.unpack_from(fmt, buf, pos)
        pos += struct.calcsize(fmt)
        return v

    def string():
        nonlocal pos
        (n,) = take("<Q")
        if n > (1 << 20):
            raise ValueError("gguf: string longer than 1 MiB")
        s = buf[pos:pos + n].decode()
        pos += n
        return s

    magic, version, ntensors, nkv = take("<IIQQ")
    if magic != GGUF_MAGIC:
        raise ValueError(f"gguf: bad magic {magic:#x}")
    if version != GGUF_VERSION:
        raise ValueError(f"gguf: unsupported version {version}")
    kvs = {}
    for _ in range(nkv):
        k = string()
        (typ,) = take("<I")
        if typ != GGUF_TYPE_STRING:
            raise ValueError(f"gguf: unexpected KV type {typ}")
        kvs[k] = string()
    if shapes is not None and len(shapes) != ntensors:
        raise ValueError(f"gguf: {ntensors} tensors in the file, {len(shapes)} in the model")
    infos = []
    for i in range(ntensors):
        string()
        (nd,) = take("<I")
        dims = take(f"<{nd}Q")
        dtype, off = take("<IQ")
        if dtype != GGUF_F32:
            raise ValueError(f"gguf: tensor {i} has type {dtype}; only F32 (0) is read here")
        if shapes is not None and tuple(dims) != tuple(shapes[i]):
            raise ValueError(f"gguf: tensor {i} shape {dims}, model {tuple(shapes[i])}")
        infos.append((dims, off))
    data_start = _align(pos)
    arrays = []
    for dims, off in infos:
        n = int(np.prod(dims)) if dims else 1
        start = data_start + off
        arrays.append(np.frombuffer(buf, np.float32, n, start).reshape(dims).copy())
    return arrays, kvs


def save_gguf(trainer, path):
    """GPT save_gguf for the model on the device."""
    write_gguf(path, [trainer.get_param(i) for i in range(trainer.num_params())])


def save_gguf_quant(trainer, path, qtype):
    """GPT save_gguf_quant for the model on the device (qtype 0, 8 or 4)."""
    write_gguf_quant(path, [trainer.get_param(i) for i in range(trainer.num_params())], qtype)


def load_gguf(trainer, path):
    """GPT load_gguf into the model on the device."""
    shapes = [trainer.param_info(i)[1] for i in range(trainer.num_params())]
    arrays, _ = read_gguf(path, shapes)
    for i, a in enumerate(arrays):
        trainer.set_param(i, a)
