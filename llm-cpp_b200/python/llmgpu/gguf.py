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

Reading decodes F32, Q8_0, Q4_0 and Q4_K tensors as the reference's load_gguf does
(src/gguf.cpp:315-353) and checks the tensor count and every shape against the model. `write_gguf_quant` writes the reference's quantized export (save_gguf_quant,
src/gguf.cpp:499-581) for qtype 0 (F32), 8 (Q8_0: per 32 values an f32 scale
max|x| / 127 + 1e-8 and 32 int8) and 4 (Q4_0: scale max|x| / 7 + 1e-8 and 16 bytes of
nibbles, value + 8, even index in the low nibble) and 12 (Q4_K: 144-byte super-blocks of
256 values, below), with the extra KV llm.quant_type; values are rounded half away from zero
as std::round does.

Q4_K super-block (encode_q4k_block, src/gguf.cpp:160-245): per 32-value sub-block j its
min mn_j and scale (max_j - mn_j) / 15; d = max scale / 63 and dmin = (largest -mn_j over
negative mins, else minus the largest min) / 63, both stored as f16 by the reference's own
f32 -> f16 rounding (round half to even, overflow saturating to 0x7BFF, its subnormal path
masked to 10 bits); 6-bit sub-block scales and mins packed into 12 bytes; each value
round((x + dmin_f * qmn_j) / (d_f * qsc_j)) clamped to 0..15 against the stored f16 scales,
value i of 64-value group g at byte 32 g + i % 32, low nibble for i % 64 < 32. A super-block
with a non-finite value is written as zeros.
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
GGUF_Q4_K = 12
_QBLK = 32


def _round_away(v):
    """std::round of float32 values (half away from zero), exact in float64."""
    v64 = v.astype(np.float64)
    return (np.sign(v64) * np.floor(np.abs(v64) + 0.5)).astype(np.float32)


def _f32_to_f16_bits(v):
    """The reference's f32 -> f16 bit conversion (src/gguf.cpp:92-119), elementwise."""
    b = np.asarray(v, np.float32).view(np.uint32).astype(np.int64)
    sign = (b >> 16) & 0x8000
    exp = ((b >> 23) & 0xFF) - 112
    mant = b & 0x7FFFFF
    out = np.zeros_like(b)
    # normal range
    half = mant >> 13
    rest = mant & 0x1FFF
    up = (rest > 0x1000) | ((rest == 0x1000) & ((half & 1) == 1))
    half = half + up
    e2 = exp + (half == 0x400)
    half = np.where(half == 0x400, 0, half)
    normal = sign | (np.clip(e2, 0, 31) << 10) | half
    normal = np.where(e2 >= 31, sign | 0x7BFF, normal)
    # subnormal range (exp in [-10, 0])
    shift = np.clip(1 - exp, 1, 31)
    m = mant | 0x800000
    hs = m >> shift
    rs = m & ((np.int64(1) << shift) - 1)
    hw = np.int64(1) << (shift - 1)
    hs = hs + ((rs > hw) | ((rs == hw) & ((hs & 1) == 1)))
    sub = sign | (hs & 0x3FF)
    out = np.where(exp >= 31, sign | 0x7BFF,
                   np.where(exp >= 1, normal, np.where(exp < -10, sign, sub)))
    return out.astype(np.uint16)


def _f16_bits_to_f32(h):
    return np.asarray(h, np.uint16).view(np.float16).astype(np.float32)


def _encode_q4k(x):
    """x: float32 [nb, 256] -> uint8 [nb, 144]."""
    f32 = np.float32
    nb = x.shape[0]
    finite = np.isfinite(x).all(axis=1)
    xs = np.where(finite[:, None], x, f32(0)).reshape(nb, 8, 32)
    mn = xs.min(axis=2)
    mx = xs.max(axis=2)
    sc_true = ((mx - mn) / f32(15)).astype(f32)
    dall_anchor = np.maximum(f32(0), sc_true.max(axis=1))
    dall = (dall_anchor / f32(63)).astype(f32)
    neg_max = np.where(mn < 0, -mn, f32(0)).max(axis=1)
    pos_max = np.where(mn >= 0, mn, f32(0)).max(axis=1)
    dmin_anchor = np.where(neg_max > 0, neg_max, -pos_max).astype(f32)
    dmin = (dmin_anchor / f32(63)).astype(f32)
    with np.errstate(divide="ignore", invalid="ignore"):
        qsc = np.where(dall_anchor[:, None] > 0,
                       np.clip(_round_away(((f32(63) * sc_true) / dall_anchor[:, None]).astype(f32)), 0, 63),
                       0).astype(np.int64)
        qmn = np.where(dmin_anchor[:, None] != 0,
                       np.clip(_round_away(((f32(63) * (-mn)) / dmin_anchor[:, None]).astype(f32)), 0, 63),
                       0).astype(np.int64)
    out = np.zeros((nb, 144), np.uint8)
    dh, mh = _f32_to_f16_bits(dall), _f32_to_f16_bits(dmin)
    out[:, 0:2] = dh[:, None].view(np.uint8).reshape(nb, 2)
    out[:, 2:4] = mh[:, None].view(np.uint8).reshape(nb, 2)
    for j in range(4):
        out[:, 4 + j] = (qsc[:, j] & 63) | ((qsc[:, j + 4] >> 4) << 6)
        out[:, 8 + j] = (qmn[:, j] & 63) | ((qmn[:, j + 4] >> 4) << 6)
        out[:, 12 + j] = (qsc[:, j + 4] & 0xF) | ((qmn[:, j + 4] & 0xF) << 4)
    dall_f, dmin_f = _f16_bits_to_f32(dh), _f16_bits_to_f32(mh)
    dj = (dall_f[:, None] * qsc.astype(f32)).astype(f32)  # [nb, 8]
    dmj = (dmin_f[:, None] * qmn.astype(f32)).astype(f32)
    xv = xs.reshape(nb, 8, 32)
    with np.errstate(divide="ignore", invalid="ignore"):
        q = _round_away(((xv + dmj[:, :, None]).astype(f32) / dj[:, :, None]).astype(f32))
    q = np.where(dj[:, :, None] != 0, np.clip(q, 0, 15), 0).astype(np.int64).reshape(nb, 4, 64)
    out[:, 16:] = (q[:, :, :32] | (q[:, :, 32:] << 4)).reshape(nb, 128).astype(np.uint8)
    return out


def _encode(a, qtype):
    x = np.ascontiguousarray(a, dtype=np.float32).ravel()
    if qtype == 0:
        return x.tobytes()
    if qtype == 12:
        x = np.concatenate([x, np.zeros((-x.size) % 256, np.float32)]).reshape(-1, 256)
        return _encode_q4k(x).tobytes()
    x = np.concatenate([x, np.zeros((-x.size) % _QBLK, np.float32)]).reshape(-1, _QBLK)
    # std::max(mx, |x|) from mx = 0 passes over NaN; a NaN quotient clamps to the top code
    mx = np.where(np.isnan(x), np.float32(0), np.abs(x)).max(axis=1)
    top = np.float32(127.0 if qtype == 8 else 7.0)
    sc = (mx / top).astype(np.float32) + np.float32(1e-8)
    with np.errstate(invalid="ignore"):
        q = _round_away((x / sc[:, None]).astype(np.float32))
    q = np.where(np.isnan(q), top, q)
    if qtype == 8:
        body = np.clip(q, -127, 127).astype(np.int8).view(np.uint8)
    else:
        q = np.clip(q, -8, 7).astype(np.int32) + 8
        body = ((q[:, 1::2] << 4) | (q[:, 0::2] & 0xF)).astype(np.uint8)
    return np.concatenate([sc[:, None].view(np.uint8), body], axis=1).tobytes()


def write_gguf_quant(path, arrays, qtype):
    """The reference's save_gguf_quant for qtype 0 (F32), 8 (Q8_0), 4 (Q4_0) or 12 (Q4_K)."""
    dtype = {0: GGUF_F32, 8: GGUF_Q8_0, 4: GGUF_Q4_0, 12: GGUF_Q4_K}.get(qtype)
    if dtype is None:
        raise ValueError(f"gguf: unknown quant type {qtype} (0, 8, 4 or 12)")
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


def _decode(buf, start, n, dtype):
    f32 = np.float32
    if dtype == GGUF_F32:
        return np.frombuffer(buf, f32, n, start).copy()
    if dtype == GGUF_Q4_K:
        nb = -(-n // 256)
        blk = np.frombuffer(buf, np.uint8, nb * 144, start).reshape(nb, 144)
        dall = _f16_bits_to_f32(blk[:, 0:2].copy().view(np.uint16)[:, 0])
        dmin = _f16_bits_to_f32(blk[:, 2:4].copy().view(np.uint16)[:, 0])
        sc8 = blk[:, 4:16].astype(np.int64)
        sc = np.empty((nb, 8), np.int64)
        mn = np.empty((nb, 8), np.int64)
        for j in range(4):  # ggml get_scale_min_k4 order
            sc[:, j], mn[:, j] = sc8[:, j] & 63, sc8[:, j + 4] & 63
            sc[:, j + 4] = (sc8[:, j + 8] & 0xF) | ((sc8[:, j] >> 6) << 4)
            mn[:, j + 4] = (sc8[:, j + 8] >> 4) | ((sc8[:, j + 4] >> 6) << 4)
        qs = blk[:, 16:].reshape(nb, 4, 32).astype(np.int64)
        q = np.concatenate([qs & 0xF, qs >> 4], axis=2).reshape(nb, 8, 32).astype(f32)
        a = (dall[:, None] * sc.astype(f32)).astype(f32)
        b = (dmin[:, None] * mn.astype(f32)).astype(f32)
        with np.errstate(invalid="ignore"):
            out = (a[:, :, None] * q).astype(f32) - b[:, :, None]
        return out.reshape(-1)[:n].astype(f32)
    nb = -(-n // _QBLK)
    width = 4 + (_QBLK if dtype == GGUF_Q8_0 else _QBLK // 2)
    blk = np.frombuffer(buf, np.uint8, nb * width, start).reshape(nb, width)
    sc = blk[:, :4].copy().view(f32)[:, 0]
    if dtype == GGUF_Q8_0:
        q = blk[:, 4:].view(np.int8).astype(f32)
    else:
        p = blk[:, 4:].astype(np.int64)
        q = np.stack([(p & 0xF) - 8, ((p >> 4) & 0xF) - 8], axis=2).reshape(nb, _QBLK).astype(f32)
    with np.errstate(invalid="ignore"):  # an inf scale times a zero code is NaN, as there
        return (q * sc[:, None]).astype(f32).reshape(-1)[:n]


def read_gguf(path, shapes=None):
    """Reads a GGUF written in the reference's layout (F32, Q8_0, Q4_0 or Q4_K tensors,
    decoded to float32); returns (arrays, kvs). With `shapes`, the tensor count and every
    shape must match (as load_gguf checks)."""
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
        if dtype not in (GGUF_F32, GGUF_Q8_0, GGUF_Q4_0, GGUF_Q4_K):
            raise ValueError(f"gguf: tensor {i} has unsupported type {dtype}")
        if shapes is not None and tuple(dims) != tuple(shapes[i]):
            raise ValueError(f"gguf: tensor {i} shape {dims}, model {tuple(shapes[i])}")
        infos.append((dims, off, dtype))
    data_start = _align(pos)
    arrays = []
    for dims, off, dtype in infos:
        n = int(np.prod(dims)) if dims else 1
        arrays.append(_decode(buf, data_start + off, n, dtype).reshape(dims))
    return arrays, kvs


def save_gguf(trainer, path):
    """GPT save_gguf for the model on the device."""
    write_gguf(path, [trainer.get_param(i) for i in range(trainer.num_params())])


def save_gguf_quant(trainer, path, qtype):
    """GPT save_gguf_quant for the model on the device (qtype 0, 8, 4 or 12)."""
    write_gguf_quant(path, [trainer.get_param(i) for i in range(trainer.num_params())], qtype)


def load_gguf(trainer, path):
    """GPT load_gguf into the model on the device."""
    shapes = [trainer.param_info(i)[1] for i in range(trainer.num_params())]
    arrays, _ = read_gguf(path, shapes)
    for i, a in enumerate(arrays):
        trainer.set_param(i, a)
