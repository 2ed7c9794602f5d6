"""Python front end of the trainer C ABI (include/tt_trainer.h).

The training step itself runs in libtinytrain.so (C++20 tt:: API on device
tensors, kernels in libttk.so). This module only marshals arguments, like the
ctypes/cgo stub a host application in another language would write.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

from . import _ttk

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "lib", "libtinytrain.so")


class ModelConfig(C.Structure):
    _fields_ = [("vocab", C.c_int64), ("dim", C.c_int64), ("layers", C.c_int64),
                ("heads", C.c_int64), ("ffn", C.c_int64), ("max_seq", C.c_int64),
                ("norm_eps", C.c_float), ("rope_theta", C.c_float)]


class AdamWConfig(C.Structure):
    _fields_ = [("lr", C.c_float), ("beta1", C.c_float), ("beta2", C.c_float),
                ("eps", C.c_float), ("weight_decay", C.c_float), ("clip_norm", C.c_float)]


# Named model configurations (GPTConfig fields, model.h:15-26).
CONFIGS = {
    # the reference's default Llama (model.h defaults / train.cpp:40)
    "llama-13m": dict(vocab=32000, dim=256, layers=6, heads=8, ffn=768, max_seq=256),
    "llama-110m": dict(vocab=32000, dim=768, layers=12, heads=12, ffn=2048, max_seq=1024),
    "llama-1b": dict(vocab=32000, dim=2048, layers=16, heads=16, ffn=5632, max_seq=2048),
}

_lib = None
P, I64, F32, U64 = C.c_void_p, C.c_int64, C.c_float, C.c_uint64
_SIGS = {
    "tt_last_error": (C.c_char_p, []),
    "tt_trainer_create": (C.c_int, [P, U64, C.c_int, P]),
    "tt_trainer_destroy": (C.c_int, [P]),
    "tt_trainer_set_stream": (C.c_int, [P, P]),
    "tt_trainer_param_count": (I64, [P]),
    "tt_trainer_init_normal": (C.c_int, [P, F32, U64]),
    "tt_trainer_set_params": (C.c_int, [P, P, I64]),
    "tt_trainer_get_params": (C.c_int, [P, P, I64]),
    "tt_trainer_get_grads": (C.c_int, [P, P, I64]),
    "tt_trainer_set_optimizer": (C.c_int, [P, P]),
    "tt_trainer_step": (C.c_int, [P, P, P, I64, I64, I64, F32, P, P]),
    "tt_trainer_step_device": (C.c_int, [P, P, P, I64, I64, I64, F32]),
    "tt_trainer_step_graph": (C.c_int, [P, P, P, I64, I64, I64, F32]),
    "tt_trainer_last_loss": (C.c_int, [P, P]),
    "tt_trainer_step_submit": (C.c_int, [P, P, P, I64, I64, I64, F32]),
    "tt_trainer_step_result": (C.c_int, [P, P, P]),
    "tt_trainer_forward_backward": (C.c_int, [P, P, P, I64, I64, P, P]),
    "tt_trainer_dist_init": (C.c_int, [P, C.c_int, C.c_int, P, I64]),
    "tt_trainer_set_collective_timeout": (C.c_int, [P, C.c_double]),
    "tt_trainer_comm_profile": (C.c_int, [P, C.c_int]),
    "tt_trainer_comm_stats": (C.c_int, [P, P, P, P, P]),
    "tt_watchdog_selftest": (C.c_int, [P, P, P, P, C.c_double, P]),
    "tt_kernel_launches": (I64, []),
    "tt_fused_attention_chains": (I64, []),
    "tt_plan_buckets": (C.c_int, [P, C.c_int, I64, P, P, P, P, P]),
    "tt_tokens_from_file": (C.c_int, [C.c_char_p, P]),
    "tt_tokens_from_host": (C.c_int, [P, I64, P]),
    "tt_tokens_count": (I64, [P]),
    "tt_tokens_destroy": (C.c_int, [P]),
    "tt_sample_windows": (C.c_int, [P, I64, I64, I64, P]),
    "tt_trainer_step_tokens": (C.c_int, [P, P, P, I64, I64, I64, F32, P, P]),
    "tt_lr_at": (F32, [F32, I64, I64, I64]),
    "tt_trainer_save": (C.c_int, [P, C.c_char_p]),
    "tt_trainer_load": (C.c_int, [P, C.c_char_p]),
}


class TrainerError(RuntimeError):
    pass


def lib():
    global _lib
    if _lib is None:
        _ttk.lib()  # libttk.so first (RTLD_GLOBAL), then the C++ layer
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: run `python -m tinytrain_b200.build`")
        _lib = C.CDLL(LIB_PATH, mode=C.RTLD_GLOBAL)
        for k, (r, a) in _SIGS.items():
            f = getattr(_lib, k)
            f.restype, f.argtypes = r, a
    return _lib


def _chk(rc, what):
    if rc != 0:
        raise TrainerError(f"{what}: {lib().tt_last_error().decode()}")


def kernel_launches() -> int:
    return int(lib().tt_kernel_launches())


def fused_attention_chains() -> int:
    """Attention-score op chains run as the fused kernel since start-up."""
    return int(lib().tt_fused_attention_chains())


_PROBE = C.CFUNCTYPE(C.c_int, C.c_void_p)


def watchdog_selftest(done, async_error, abort, timeout_s):
    """Runs the collective watchdog's wait loop on Python probes (callables
    without arguments returning int); returns its outcome (0 done, 1 error,
    2 timeout)."""
    cbs = [_PROBE(lambda _c, f=f: int(f())) for f in (done, async_error, abort)]
    out = C.c_int(-1)
    _chk(lib().tt_watchdog_selftest(C.cast(cbs[0], P), C.cast(cbs[1], P), C.cast(cbs[2], P),
                                    None, float(timeout_s), C.byref(out)), "watchdog selftest")
    return out.value


def set_stream(stream_handle: int):
    _chk(lib().tt_trainer_set_stream(None, stream_handle), "set_stream")


class Trainer:
    """GPTModel + AdamW on one GPU (optionally one rank of a DP job)."""

    def __init__(self, config, seed=42, host_init=True, norm_eps=1e-5, rope_theta=10000.0):
        if isinstance(config, str):
            config = CONFIGS[config]
        self.cfg = dict(config)
        mc = ModelConfig(self.cfg["vocab"], self.cfg["dim"], self.cfg["layers"], self.cfg["heads"],
                         self.cfg["ffn"], self.cfg["max_seq"], norm_eps, rope_theta)
        h = C.c_void_p()
        _chk(lib().tt_trainer_create(C.byref(mc), seed, int(host_init), C.byref(h)), "create")
        self.h = h
        self.n_params = int(lib().tt_trainer_param_count(self.h))

    def close(self):
        if self.h:
            _chk(lib().tt_trainer_destroy(self.h), "destroy")
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def init_normal(self, std=0.02, seed=0):
        _chk(lib().tt_trainer_init_normal(self.h, std, seed), "init_normal")

    def set_params(self, flat):
        flat = np.ascontiguousarray(flat, np.float32)
        _chk(lib().tt_trainer_set_params(self.h, flat.ctypes.data, flat.size), "set_params")

    def get_params(self):
        out = np.empty(self.n_params, np.float32)
        _chk(lib().tt_trainer_get_params(self.h, out.ctypes.data, out.size), "get_params")
        return out

    def get_grads(self):
        out = np.empty(self.n_params, np.float32)
        _chk(lib().tt_trainer_get_grads(self.h, out.ctypes.data, out.size), "get_grads")
        return out

    def set_optimizer(self, lr=3e-4, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1, clip=1.0):
        c = AdamWConfig(lr, betas[0], betas[1], eps, weight_decay, clip)
        _chk(lib().tt_trainer_set_optimizer(self.h, C.byref(c)), "set_optimizer")

    def step(self, idx, targets, B, T, n_micro=1, lr=3e-4):
        """Host ids (int64, n_micro*B*T); returns (loss, grad_norm)."""
        idx = np.ascontiguousarray(idx, np.int64)
        targets = np.ascontiguousarray(targets, np.int64)
        loss, gn = C.c_float(0), C.c_float(0)
        _chk(lib().tt_trainer_step(self.h, idx.ctypes.data, targets.ctypes.data, B, T, n_micro,
                                   lr, C.byref(loss), C.byref(gn)), "step")
        return loss.value, gn.value

    def step_submit(self, idx, targets, B, T, n_micro=1, lr=3e-4):
        """Enqueue one step on host ids and return at once (collect it with
        step_result; at most two in flight)."""
        idx = np.ascontiguousarray(idx, np.int64)
        targets = np.ascontiguousarray(targets, np.int64)
        _chk(lib().tt_trainer_step_submit(self.h, idx.ctypes.data, targets.ctypes.data, B, T,
                                          n_micro, lr), "step_submit")

    def step_result(self):
        """(loss, grad_norm) of the oldest submitted step, waiting for it."""
        loss, gn = C.c_float(0), C.c_float(0)
        _chk(lib().tt_trainer_step_result(self.h, C.byref(loss), C.byref(gn)), "step_result")
        return loss.value, gn.value

    def step_device(self, idx_ptr, tgt_ptr, B, T, n_micro=1, lr=3e-4):
        _chk(lib().tt_trainer_step_device(self.h, idx_ptr, tgt_ptr, B, T, n_micro, lr),
             "step_device")

    def step_graph(self, idx_ptr, tgt_ptr, B, T, n_micro=1, lr=3e-4):
        """step_device replayed from a CUDA graph (one GPU): the first call with
        these pointers and sizes runs eagerly, the second records and launches the
        graph, later ones launch it. The ids must be in the same device buffers
        each call."""
        _chk(lib().tt_trainer_step_graph(self.h, idx_ptr, tgt_ptr, B, T, n_micro, lr),
             "step_graph")

    def last_loss(self):
        v = C.c_float(0)
        _chk(lib().tt_trainer_last_loss(self.h, C.byref(v)), "last_loss")
        return v.value

    def forward_backward(self, idx, targets, B, T, want_logits=False):
        idx = np.ascontiguousarray(idx, np.int64)
        targets = np.ascontiguousarray(targets, np.int64)
        loss = C.c_float(0)
        logits = np.empty((B * T, self.cfg["vocab"]), np.float32) if want_logits else None
        _chk(lib().tt_trainer_forward_backward(
            self.h, idx.ctypes.data, targets.ctypes.data, B, T, C.byref(loss),
            None if logits is None else logits.ctypes.data), "forward_backward")
        return loss.value, logits

    def set_collective_timeout(self, seconds):
        """Deadline for a distributed step's collectives; on an overrun or an
        asynchronous NCCL error the communicator is aborted and the step fails."""
        _chk(lib().tt_trainer_set_collective_timeout(self.h, float(seconds)), "collective timeout")

    def comm_profile(self, on=True):
        _chk(lib().tt_trainer_comm_profile(self.h, int(on)), "comm profile")

    def comm_stats(self):
        """(all-reduce ms summed over buckets, exposed tail ms summed over
        steps, all-reduce count, step count) since the last read."""
        a, t, n, k = C.c_double(0), C.c_double(0), C.c_int64(0), C.c_int64(0)
        _chk(lib().tt_trainer_comm_stats(self.h, C.byref(a), C.byref(t), C.byref(n), C.byref(k)),
             "comm stats")
        return a.value, t.value, n.value, k.value

    def dist_init(self, rank, world, uid: bytes, bucket_bytes=64 << 20):
        buf = (C.c_ubyte * 128).from_buffer_copy(uid)
        _chk(lib().tt_trainer_dist_init(self.h, rank, world, buf, bucket_bytes), "dist_init")

    def step_tokens(self, tokens: "TokenStream", starts, B, T, n_micro=1, lr=3e-4):
        """One step on windows of a device token stream; `starts` are this
        rank's n_micro*B window starts. Returns (loss, grad_norm)."""
        st = np.ascontiguousarray(starts, np.int64)
        loss, gn = C.c_float(0), C.c_float(0)
        _chk(lib().tt_trainer_step_tokens(self.h, tokens.h, st.ctypes.data, B, T, n_micro, lr,
                                          C.byref(loss), C.byref(gn)), "step_tokens")
        return loss.value, gn.value

    def save(self, path):
        _chk(lib().tt_trainer_save(self.h, os.fsencode(path)), "save")

    def load(self, path):
        _chk(lib().tt_trainer_load(self.h, os.fsencode(path)), "load")


class TokenStream:
    """An int32 token stream held in device memory (apps/prepare_data.cpp's
    file format), from a file path or a host array."""

    def __init__(self, path=None, host=None):
        h = C.c_void_p()
        if path is not None:
            _chk(lib().tt_tokens_from_file(os.fsencode(path), C.byref(h)), "tokens")
        else:
            self._host = np.ascontiguousarray(host, np.int32)
            _chk(lib().tt_tokens_from_host(self._host.ctypes.data, self._host.size, C.byref(h)),
                 "tokens")
        self.h = h.value

    def __len__(self):
        return int(lib().tt_tokens_count(self.h))

    def close(self):
        if self.h:
            lib().tt_tokens_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class WindowSampler:
    """The reference's window sampler (apps/train.cpp:145-153, 225-232): its
    xorshift64* stream seeded with `seed` (train.cpp passes seed + 999)."""

    def __init__(self, seed):
        self.state = C.c_uint64(seed)

    def draw(self, ntok, T, count):
        out = np.empty(count, np.int64)
        _chk(lib().tt_sample_windows(C.byref(self.state), ntok, T, count, out.ctypes.data),
             "sample_windows")
        return out


def lr_at(base_lr, step, warmup, total_steps) -> float:
    """apps/train.cpp:214-222 learning rate for global step `step`."""
    return float(lib().tt_lr_at(base_lr, step, warmup, total_steps))


def plan_buckets(sizes, bucket_bytes):
    """(offsets, bucket_of_param, [(bucket_offset, bucket_len)]) of the DP
    gradient arena for parameters of these sizes (host-only computation)."""
    n = len(sizes)
    sz = np.ascontiguousarray(sizes, np.int64)
    offs = np.zeros(n, np.int64)
    ids = np.zeros(n, np.int32)
    boff = np.zeros(max(n, 1), np.int64)
    bcnt = np.zeros(max(n, 1), np.int64)
    nb = C.c_int(0)
    _chk(lib().tt_plan_buckets(sz.ctypes.data, n, bucket_bytes, offs.ctypes.data, ids.ctypes.data,
                               boff.ctypes.data, bcnt.ctypes.data, C.byref(nb)), "plan_buckets")
    return offs, ids, list(zip(boff[:nb.value].tolist(), bcnt[:nb.value].tolist()))


def dist_unique_id() -> bytes:
    buf = (C.c_ubyte * 128)()
    _ttk.call("ttk_dist_unique_id", buf)
    return bytes(buf)
