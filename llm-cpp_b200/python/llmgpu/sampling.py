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


class MT19937:
    """std::mt19937: the standard 32-bit Mersenne Twister with its standard seeding, as one
    stream of outputs (the reference's GPT::generate draws every token from one stream)."""

    def __init__(self, seed):
        self.bg = np.random.MT19937(0)
        self.bg._legacy_seeding(int(seed) & 0xFFFFFFFF)  # init_genrand, as std::mt19937(seed)

    def next_u32(self):
        return int(self.bg.random_raw())

    def canonical(self):
        """generate_canonical<double, 53> (libstdc++): two outputs, low word first."""
        g1, g2 = self.next_u32(), self.next_u32()
        p = (float(g1) + float(g2) * 4294967296.0) / 18446744073709551616.0
        return p if p < 1.0 else float(np.nextafter(1.0, 0.0))

    def uniform_int(self, a, b):
        """std::uniform_int_distribution<int>(a, b) over a 32-bit engine (libstdc++): Lemire's
        multiply-and-reject downscaling of one output (more only on a rejection)."""
        r = b - a + 1
        if r == 1 << 32:
            return self.next_u32() + a
        prod = self.next_u32() * r
        low = prod & 0xFFFFFFFF
        if low < r:
            threshold = ((1 << 32) - r) % r
            while low < threshold:
                prod = self.next_u32() * r
                low = prod & 0xFFFFFFFF
        return (prod >> 32) + a


def _discrete_draw(weights, p):
    w = [float(v) for v in weights]
    s = 0.0
    for v in w:
        s += v
    cp, acc = [], 0.0
    for v in w:
        acc += v / s
        cp.append(acc)
    cp[-1] = 1.0
    return int(np.searchsorted(np.asarray(cp), p, side="left"))


def _discrete(weights, seed):
    """std::discrete_distribution drawn once from a fresh std::mt19937(seed)."""
    return _discrete_draw(weights, MT19937(seed).canonical())


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


def generate(forward_logits, prompt, max_new_tokens, max_seq, vocab, temperature=0.0, top_k=0,
             top_p=1.0, rep_penalty=1.0, seed=42, global_seed=42, eos_id=None, stop_ids=()):
    """GPT::generate (src/model.cpp:393-474) over a logits function (tokens [1, T] -> [1, V]):

    - the logits of the last position over the last max_seq tokens (zeros, i.e. uniform,
      for an empty prompt), then the repetition penalty;
    - temperature 0: the first maximum;
    - otherwise the logits are divided by the temperature, then
      * top_p < 1 with top_k == 0: sample_top_p with the global seed (every token draws from
        a fresh std::mt19937(global_seed), as the reference's sample_top_p does);
      * top_k > 0: one of the k largest logits, uniformly (std::uniform_int_distribution on
        the generator stream);
      * else: softmax, then std::discrete_distribution on the generator stream;
    - the generator stream is one std::mt19937(seed) for the whole call (42 in the
      reference).
    Among equal logits, the top-k order here is index order (std::partial_sort leaves it
    unspecified). Stops early at eos_id / stop_ids (generate_with_stop's rule)."""
    out = [int(t) for t in prompt]
    rng = MT19937(seed)
    last = np.asarray(forward_logits(np.asarray(out[-max_seq:], np.int32)[None, :])[0], _F32) \
        if out else np.zeros(int(vocab), _F32)
    for step in range(int(max_new_tokens)):
        cur = np.array(last, _F32)
        if rep_penalty != 1.0:
            cur = apply_repetition_penalty(cur, out, rep_penalty)
        if temperature == 0.0:
            nxt = sample_greedy(cur)
        else:
            if temperature != 1.0:
                cur = (cur / _F32(temperature)).astype(_F32)
            if top_p < 1.0 and top_k == 0:
                nxt = sample_top_p_seeded(cur, top_p, 1.0, global_seed)
            elif top_k > 0:
                idx = np.argsort(-cur, kind="stable")[:top_k]
                nxt = int(idx[rng.uniform_int(0, top_k - 1)])
            else:
                nxt = _discrete_draw(_softmax32(cur), rng.canonical())
        out.append(nxt)
        if eos_id is not None and should_stop(nxt, eos_id, stop_ids):
            break
        if step + 1 >= max_new_tokens:
            break
        last = np.asarray(forward_logits(np.asarray(out[-max_seq:], np.int32)[None, :])[0], _F32)
    return out
