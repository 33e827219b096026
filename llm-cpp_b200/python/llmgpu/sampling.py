"""Token samplers of the reference (src/sampling.cpp), with the same arithmetic and random
stream, so a seeded pick is the reference's pick:

- logits are divided by the temperature, exponentiated against their maximum and normalised
  in float32 with sequential sums, as the reference's loops do;
- `std::mt19937(seed)` is the standard 32-bit Mersenne Twister with its standard seeding;
- `std::discrete_distribution` (libstdc++): the weights normalised in double, their running
  sum with the last entry set to 1, one `generate_canonical<double, 53>` draw
  ((first 32-bit output + second * 2^32) / 2^64) and the first running sum not below it;
- top-k takes the k largest (temperature-scaled) logits, top-p the most probable tokens
  until their probability reaches p, both renormalised before the draw.
Also `apply_repetition_penalty`, `apply_freq_presence`, `apply_logit_bias` and
`should_stop`, as there.
"""
import numpy as np

_F32 = np.float32


def _mt_draw(seed):
    bg = np.random.MT19937(0)
    bg._legacy_seeding(int(seed) & 0xFFFFFFFF)  # init_genrand, as std::mt19937(seed)
    g1, g2 = (int(v) for v in bg.random_raw(2))
    p = (float(g1) + float(g2) * 4294967296.0) / 18446744073709551616.0
    return p if p < 1.0 else float(np.nextafter(1.0, 0.0))


def _discrete(weights, seed):
    w = [float(v) for v in weights]
    s = 0.0
    for v in w:
        s += v
    cp, acc = [], 0.0
    for v in w:
        acc += v / s
        cp.append(acc)
    cp[-1] = 1.0
    return int(np.searchsorted(np.asarray(cp), _mt_draw(seed), side="left"))


def _softmax32(l):
    l = np.asarray(l, _F32)
    e = np.exp(l - l.max()).astype(_F32)
    s = np.add.accumulate(e, dtype=_F32)[-1]
    return (e / s).astype(_F32)


def sample_greedy(logits):
    return int(np.argmax(np.asarray(logits, _F32)))


def sample_temperature_seeded(logits, temp, seed):
    l = (np.asarray(logits, _F32) / _F32(temp)).astype(_F32)
    return _discrete(_softmax32(l), seed)


def sample_top_k_seeded(logits, k, temp, seed):
    tmp = (np.asarray(logits, _F32) / _F32(temp)).astype(_F32)
    idx = np.argsort(-tmp, kind="stable")[:k]
    return int(idx[_discrete(_softmax32(tmp[idx]), seed)])


def sample_top_p_seeded(logits, p, temp, seed):
    l = _softmax32((np.asarray(logits, _F32) / _F32(temp)).astype(_F32))
    idx = np.argsort(-l, kind="stable")
    cum = np.add.accumulate(l[idx], dtype=_F32)
    hit = np.nonzero(cum >= _F32(p))[0]
    last = int(hit[0]) if hit.size else len(idx) - 1
    filt = l[idx[:last + 1]]
    s = np.add.accumulate(filt, dtype=_F32)[-1]
    return int(idx[_discrete((filt / s).astype(_F32), seed)])


def apply_repetition_penalty(logits, generated, penalty):
    out = np.array(logits, _F32)
    for i in generated:
        if 0 <= i < out.size:
            out[i] = out[i] / _F32(penalty) if out[i] > 0 else out[i] * _F32(penalty)
    return out


def apply_freq_presence(logits, generated, freq_penalty, pres_penalty):
    out = np.array(logits, _F32)
    ids, counts = np.unique([i for i in generated if 0 <= i < out.size], return_counts=True)
    for i, n in zip(ids, counts):
        out[i] -= _F32(freq_penalty) * _F32(n) + _F32(pres_penalty)
    return out


def apply_logit_bias(logits, bias):
    out = np.array(logits, _F32)
    for i, b in bias.items():
        if 0 <= i < out.size:
            out[i] += _F32(b)
    return out


def should_stop(next_id, eos_id, stop_ids=()):
    return next_id == eos_id or next_id in stop_ids


def generate(forward_logits, prompt, max_new_tokens, max_seq, temperature=0.0, top_k=0,
             top_p=1.0, rep_penalty=1.0, seed=42, eos_id=None, stop_ids=()):
    """GPT::generate's loop over a logits function (tokens [1, T] -> [1, V]): per new token,
    the logits of the last position over the last max_seq tokens, the repetition penalty,
    then greedy (temperature 0), top-k (k > 0), top-p (p < 1) or temperature sampling.
    Token i draws with seed + i (GPT::generate draws every token from one std::mt19937
    stream instead). Stops early at eos_id / stop_ids."""
    out = [int(t) for t in prompt]
    for i in range(int(max_new_tokens)):
        ctx = np.asarray(out[-max_seq:] or [0], np.int32)[None, :]
        l = np.asarray(forward_logits(ctx)[0], _F32)
        if rep_penalty != 1.0:
            l = apply_repetition_penalty(l, out, rep_penalty)
        if temperature == 0.0:
            nxt = sample_greedy(l)
        elif top_k > 0:
            nxt = sample_top_k_seeded(l, top_k, temperature, seed + i)
        elif top_p < 1.0:
            nxt = sample_top_p_seeded(l, top_p, temperature, seed + i)
        else:
            nxt = sample_temperature_seeded(l, temperature, seed + i)
        out.append(nxt)
        if eos_id is not None and should_stop(nxt, eos_id, stop_ids):
            break
    return out
