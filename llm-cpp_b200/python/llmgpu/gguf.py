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

Reading accepts F32 tensors only (the reference's Q8_0 / Q4_0 / Q4_K storage is not read
here) and checks the tensor count and every shape against the model.
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


def load_gguf(trainer, path):
    """GPT load_gguf into the model on the device."""
    shapes = [trainer.param_info(i)[1] for i in range(trainer.num_params())]
    arrays, _ = read_gguf(path, shapes)
    for i, a in enumerate(arrays):
        trainer.set_param(i, a)
