"""Python mirror of the reference's training interface over libllmgpu.so.

`GPT` + `Trainer` follow the names and argument meaning of llm::GPT / llm::Trainer /
llm::AdamW (include/llm/model.h, include/llm/trainer.h, include/llm/optimizer.h); all
compute runs in the CUDA kernels behind the C ABI. Errors raise `LlmgpuError` with the
library's message (the reference asserts or throws at the same points).
"""
import ctypes
import math

import numpy as np

from ._abi_decl import LlmgpuConfig
from ._lib import load

OK, SKIPPED = 0, 1


class LlmgpuError(RuntimeError):
    pass


def make_config(vocab_size=50257, n_layers=12, n_heads=12, n_embd=768, block_size=1024,
                weight_tying=True, use_rmsnorm=False, use_mamba=False, d_inner=0, d_state=16,
                dt_rank=0, conv_kernel=4, ffn_swiglu=False, ffn_hidden=0, rope_qk=False,
                rope_theta=10000.0, moe_experts=0, moe_top_k=2, moe_aux_coef=0.01,
                pos_encoding=0, rope_scaling=1.0, rope_mode=0, yarn_alpha=1.0, yarn_beta=32.0):
    lib = load()
    c = LlmgpuConfig()
    lib.llmgpu_config_default(ctypes.byref(c))
    for k, v in dict(vocab_size=vocab_size, n_layers=n_layers, n_heads=n_heads, n_embd=n_embd,
                     block_size=block_size, weight_tying=int(weight_tying),
                     use_rmsnorm=int(use_rmsnorm), use_mamba=int(use_mamba), d_inner=d_inner,
                     d_state=d_state, dt_rank=dt_rank, conv_kernel=conv_kernel,
                     ffn_swiglu=int(ffn_swiglu), ffn_hidden=ffn_hidden, rope_qk=int(rope_qk),
                     rope_theta=rope_theta, moe_experts=moe_experts, moe_top_k=moe_top_k,
                     moe_aux_coef=moe_aux_coef, pos_encoding=int(pos_encoding),
                     rope_scaling=rope_scaling, rope_mode=rope_mode, yarn_alpha=yarn_alpha,
                     yarn_beta=yarn_beta).items():
        setattr(c, k, v)
    return c


def unique_id():
    buf = ctypes.create_string_buffer(128)
    rc = load().llmgpu_get_unique_id(buf)
    if rc != 0:
        raise LlmgpuError(f"llmgpu_get_unique_id failed ({rc})")
    return buf.raw


class Trainer:
    """Device training context: GPT parameters + AdamW state + Trainer counters."""

    def __init__(self, cfg: LlmgpuConfig, max_batch, max_seq, rank=0, world=1, uid=None):
        self.lib = load()
        self.cfg = cfg
        uidbuf = ctypes.create_string_buffer(uid, 128) if uid is not None else None
        self.h = self.lib.llmgpu_create(ctypes.byref(cfg), max_batch, max_seq, rank, world,
                                        uidbuf)
        if not self.h:
            raise LlmgpuError(self.lib.llmgpu_last_error(None).decode())
        self.max_batch, self.max_seq = max_batch, max_seq
        self._lr = 3e-4  # the library's AdamW default
        self._last_good = None

    # ------------------------------------------------------------------ lifecycle
    def close(self):
        if getattr(self, "h", None):
            self.lib.llmgpu_destroy(self.h)
            self.h = None

    def __del__(self):
        self.close()

    def _err(self, what, rc):
        msg = self.lib.llmgpu_last_error(self.h)
        raise LlmgpuError(f"{what} failed ({rc}): {msg.decode() if msg else ''}")

    # ------------------------------------------------------------------ hyper-parameters
    def set_adamw(self, lr=3e-4, b1=0.9, b2=0.95, eps=1e-8, wd=0.1):
        self.lib.llmgpu_set_adamw(self.h, lr, b1, b2, eps, wd)
        self._lr = float(lr)

    def set_lr(self, lr):
        self.lib.llmgpu_set_lr(self.h, lr)
        self._lr = float(lr)

    def get_lr(self):
        """Optimizer::get_lr: the learning rate last set through this object."""
        return self._lr

    def snapshot_params(self):
        """Trainer::snapshot_params (src/trainer.cpp:234-238): keep a host copy of every
        parameter as the last good state."""
        self._last_good = [self.get_param(i) for i in range(self.num_params())]

    def rollback_if_nonfinite(self, loss):
        """Trainer::rollback_if_nonfinite (src/trainer.cpp:239-246): if `loss` is not finite
        and a snapshot exists, restore the snapshot's parameters and halve the learning rate.
        Returns whether it rolled back. (Adam's moments are left as they are, as there.)"""
        if math.isfinite(loss) or self._last_good is None:
            return False
        for i, p in enumerate(self._last_good):
            self.set_param(i, p)
        self.set_lr(self._lr * 0.5)
        return True

    def set_train(self, grad_clip=1.0, grad_accum_steps=1, label_smoothing=0.0):
        rc = self.lib.llmgpu_set_train(self.h, grad_clip, grad_accum_steps, label_smoothing)
        if rc:
            self._err("set_train", rc)

    def set_loss_scale(self, scale):
        """TrainConfig::loss_scale: loss gradient times `scale`, parameter gradients divided
        by it before the clip."""
        rc = self.lib.llmgpu_set_loss_scale(self.h, scale)
        if rc:
            self._err("set_loss_scale", rc)

    def set_comm_timeout(self, seconds):
        """Bound (seconds) on any wait for a collective; past it the communicator is aborted
        and the step raises LlmgpuError (LLMGPU_E_NCCL)."""
        rc = self.lib.llmgpu_set_comm_timeout(self.h, float(seconds))
        if rc:
            self._err("set_comm_timeout", rc)

    def abort_comm(self):
        """Ends the communicator between steps once a peer is known to be gone (see
        llmgpu.dist.PeerWatch); later steps raise LlmgpuError without launching."""
        rc = self.lib.llmgpu_abort_comm(self.h)
        if rc:
            self._err("abort_comm", rc)

    def set_graph(self, enable):
        self.lib.llmgpu_set_graph(self.h, int(enable))

    # ------------------------------------------------------------------ steps
    def train_step(self, tokens):
        """tokens: int32 array [B, T]. Returns (loss, grad_norm, skipped)."""
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        B, T = t.shape
        loss, gn = ctypes.c_float(), ctypes.c_float()
        rc = self.lib.llmgpu_train_step(self.h, t.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)),
                                        B, T, ctypes.byref(loss), ctypes.byref(gn))
        if rc < 0:
            self._err("train_step", rc)
        return loss.value, gn.value, rc == SKIPPED

    def train_step_accum(self, tokens):
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        B, T = t.shape
        loss, stepped = ctypes.c_float(), ctypes.c_int()
        rc = self.lib.llmgpu_train_step_accum(
            self.h, t.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), B, T, ctypes.byref(loss),
            ctypes.byref(stepped))
        if rc < 0:
            self._err("train_step_accum", rc)
        return loss.value, bool(stepped.value), rc == SKIPPED

    def train_step_device(self, dev_ptr, B, T):
        loss, gn = ctypes.c_float(), ctypes.c_float()
        rc = self.lib.llmgpu_train_step_device(self.h, ctypes.c_void_p(dev_ptr), B, T,
                                               ctypes.byref(loss), ctypes.byref(gn))
        if rc < 0:
            self._err("train_step_device", rc)
        return loss.value, gn.value, rc == SKIPPED

    def eval_loss(self, tokens):
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        B, T = t.shape
        loss = ctypes.c_float()
        rc = self.lib.llmgpu_eval_loss(self.h, t.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)),
                                       B, T, ctypes.byref(loss))
        if rc < 0:
            self._err("eval_loss", rc)
        return loss.value

    def forward_logits(self, tokens):
        """tokens int32 [B, T] -> float32 [B, V]: the logits of each sequence's last position
        (GPT::forward, row T-1)."""
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        B, T = t.shape
        out = np.empty((B, self.cfg.vocab_size), np.float32)
        n = self.lib.llmgpu_forward_logits(self.h, t.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)),
                                           B, T, out.ctypes.data_as(ctypes.POINTER(ctypes.c_float)),
                                           out.size)
        if n < 0:
            self._err("forward_logits", n)
        return out

    def forward_logits_all(self, tokens):
        """tokens int32 [B, T] -> float32 [B, T, V]: the logits of every position
        (GPT::forward)."""
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        B, T = t.shape
        out = np.empty((B, T, self.cfg.vocab_size), np.float32)
        n = self.lib.llmgpu_forward_logits_all(
            self.h, t.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), B, T,
            out.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), out.size)
        if n < 0:
            self._err("forward_logits_all", n)
        return out

    # ------------------------------------------------------------------ KV-cached decoding
    def decode_reset(self, B):
        """Starts B empty sequences in the device KV caches."""
        rc = self.lib.llmgpu_decode_reset(self.h, int(B))
        if rc:
            self._err("decode_reset", rc)

    def decode_prefill(self, tokens):
        """tokens int32 [B, T] -> float32 [B, V]: runs the prompts, keeps their keys and
        values, returns each prompt's last-position logits."""
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        B, T = t.shape
        out = np.empty((B, self.cfg.vocab_size), np.float32)
        n = self.lib.llmgpu_decode_prefill(self.h, t.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)),
                                           B, T, out.ctypes.data_as(ctypes.POINTER(ctypes.c_float)),
                                           out.size)
        if n < 0:
            self._err("decode_prefill", n)
        return out

    def decode_step(self, tokens):
        """tokens int32 [B] (one per sequence) -> float32 [B, V]: the logits of the position
        the tokens were appended at."""
        t = np.ascontiguousarray(tokens, dtype=np.int32).ravel()
        out = np.empty((t.size, self.cfg.vocab_size), np.float32)
        n = self.lib.llmgpu_decode_step(self.h, t.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)),
                                        t.size, out.ctypes.data_as(ctypes.POINTER(ctypes.c_float)),
                                        out.size)
        if n < 0:
            self._err("decode_step", n)
        return out

    def decode_position(self):
        return self.lib.llmgpu_decode_position(self.h)

    def decode_supported(self):
        c = self.cfg
        return not (c.use_mamba or c.moe_experts or c.ffn_swiglu or c.rope_qk)

    def generate(self, prompt, max_new_tokens, use_cache=True, **sampling_args):
        """GPT::generate (src/model.cpp:393-474) on the device: greedy by default; the
        reference's temperature / top-k / top-p / repetition-penalty options and its one
        std::mt19937(42) stream, as in llmgpu.sampling.generate. With use_cache (and a
        configuration the KV-cached decode covers) each new token runs one decode step against
        the cached keys and values, as the reference's incremental forward does; otherwise, and
        once the window slides past max_seq, the forward re-runs over the last max_seq tokens.
        Returns prompt + generated ids."""
        from . import sampling
        fwd = self.forward_logits
        if use_cache and self.decode_supported():
            fwd = _CachedForward(self)
        return sampling.generate(fwd, prompt, max_new_tokens, self.max_seq,
                                 self.cfg.vocab_size, **sampling_args)

    # ------------------------------------------------------------------ parameters
    def num_params(self):
        return self.lib.llmgpu_num_params(self.h)

    def num_parameters(self):
        return self.lib.llmgpu_num_parameters(self.h)

    def param_info(self, i):
        name = ctypes.create_string_buffer(128)
        shape = (ctypes.c_int64 * 4)()
        nd = self.lib.llmgpu_param_info(self.h, i, name, 128, shape)
        if nd < 0:
            self._err("param_info", nd)
        return name.value.decode(), tuple(shape[j] for j in range(nd))

    def _get(self, fn, i):
        _, shape = self.param_info(i)
        out = np.empty(int(np.prod(shape)), np.float32)
        n = fn(self.h, i, out.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), out.size)
        if n < 0:
            self._err("get", n)
        return out.reshape(shape)

    def get_param(self, i):
        return self._get(self.lib.llmgpu_get_param, i)

    def get_grad(self, i):
        return self._get(self.lib.llmgpu_get_grad, i)

    def get_adam_state(self, i):
        _, shape = self.param_info(i)
        m = np.empty(int(np.prod(shape)), np.float32)
        v = np.empty_like(m)
        n = self.lib.llmgpu_get_adam_state(self.h, i, m.ctypes.data_as(ctypes.POINTER(ctypes.c_float)),
                                           v.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), m.size)
        if n < 0:
            self._err("get_adam_state", n)
        return m.reshape(shape), v.reshape(shape)

    def set_param(self, i, a):
        a = np.ascontiguousarray(a, np.float32).ravel()
        rc = self.lib.llmgpu_set_param(self.h, i, a.ctypes.data_as(ctypes.POINTER(ctypes.c_float)),
                                       a.size)
        if rc:
            self._err("set_param", rc)

    def params(self):
        return [self.get_param(i) for i in range(self.num_params())]

    def grads(self):
        return [self.get_grad(i) for i in range(self.num_params())]

    def names(self):
        return [self.param_info(i)[0] for i in range(self.num_params())]

    # ------------------------------------------------------------------ checkpoints
    def save_binary(self, path):
        rc = self.lib.llmgpu_save_binary(self.h, path.encode())
        if rc:
            self._err("save_binary", rc)

    def load_binary(self, path):
        rc = self.lib.llmgpu_load_binary(self.h, path.encode())
        if rc:
            self._err("load_binary", rc)

    def save_train_state(self, prefix):
        rc = self.lib.llmgpu_save_train_state(self.h, prefix.encode())
        if rc:
            self._err("save_train_state", rc)

    def load_train_state(self, prefix):
        rc = self.lib.llmgpu_load_train_state(self.h, prefix.encode())
        if rc:
            self._err("load_train_state", rc)

    # ------------------------------------------------------------------ counters
    def step(self):
        return self.lib.llmgpu_step(self.h)

    def set_step(self, s):
        self.lib.llmgpu_set_step(self.h, s)

    def skipped_steps(self):
        return self.lib.llmgpu_skipped_steps(self.h)

    def last_loss(self):
        return self.lib.llmgpu_last_loss(self.h)

    def last_grad_norm(self):
        return self.lib.llmgpu_last_grad_norm(self.h)

    def last_timings(self):
        t = (ctypes.c_float * 6)()
        self.lib.llmgpu_last_timings(self.h, t)
        return dict(zip(["forward", "loss", "backward", "allreduce", "optimizer", "total"], list(t)))

    def last_launches(self):
        return self.lib.llmgpu_last_launches(self.h)

    def stream(self):
        return self.lib.llmgpu_stream(self.h)

    def set_profile(self, on):
        self.lib.llmgpu_set_profile(self.h, int(on))

    def gemm_stats(self, reset=False):
        f, ms, n = ctypes.c_double(), ctypes.c_double(), ctypes.c_int()
        self.lib.llmgpu_gemm_stats(self.h, ctypes.byref(f), ctypes.byref(ms), ctypes.byref(n),
                                   int(reset))
        return f.value, ms.value, n.value

    def gemm_last_step(self):
        """Per GEMM launch of the last profiled step: (shapes [n, 6] = M, N, K of the first and
        second product, device ms [n])."""
        n = self.lib.llmgpu_gemm_last_step(self.h, None, None, 0)
        shapes = np.zeros((max(n, 0), 6), np.int32)
        ms = np.zeros(max(n, 0), np.float32)
        if n > 0:
            self.lib.llmgpu_gemm_last_step(
                self.h, shapes.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)),
                ms.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), n)
        return shapes, ms

    def moe_routing(self, layer, B, T, k):
        """Top-k expert indices [B*T, k] chosen by block `layer` in the last forward pass."""
        out = np.empty((B * T, k), np.int32)
        n = self.lib.llmgpu_moe_routing(self.h, layer, out.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)),
                                        out.size)
        if n < 0:
            self._err("moe_routing", n)
        return out


class _CachedForward:
    """Logits of the last position of a token window, through the KV caches: a window that
    extends the previous one by one token is one decode step, any other window a prefill."""

    def __init__(self, tr):
        self.tr = tr
        self.seen = None

    def __call__(self, ctx):
        toks = [int(t) for t in np.asarray(ctx)[0]]
        if (self.seen is not None and len(toks) == len(self.seen) + 1
                and toks[:-1] == self.seen):
            out = self.tr.decode_step(np.asarray(toks[-1:], np.int32))
        else:
            out = self.tr.decode_prefill(np.asarray([toks], np.int32))
        self.seen = toks
        return out

