"""Python face of include/mle_engine.h: a training session of one benchmark
configuration running on the native runtime.

    s = Session.encoder(batch=32, seq_len=128, d_model=256, heads=8, ffn=1024,
                        layers=2, vocab=4096, seed=0)
    s.inputs["tokens"][:] = ids          # pinned host staging (numpy views)
    s.inputs["targets"][:] = next_ids
    loss = s.step()                       # H2D, fwd, bwd, clip, AdamW, D2H

Everything runs in libmle_engine.so; this module only marshals arguments.
"""
from __future__ import annotations

import ctypes

import numpy as np

from ._lib import MLEError, engine

MLP, ENCODER, ENCDEC, UNET = 1, 2, 3, 4
KEYGRAD_REFERENCE, KEYGRAD_TRUE = 0, 1


class SessionDesc(ctypes.Structure):
    _fields_ = [
        ("config", ctypes.c_int), ("batch", ctypes.c_int),
        ("in_features", ctypes.c_int), ("hidden", ctypes.c_int), ("classes", ctypes.c_int),
        ("seq_len", ctypes.c_int), ("d_model", ctypes.c_int), ("heads", ctypes.c_int), ("ffn", ctypes.c_int),
        ("layers", ctypes.c_int), ("vocab", ctypes.c_int),
        ("fused_attention", ctypes.c_int), ("key_grad_mode", ctypes.c_int),
        ("lr", ctypes.c_float), ("adamw", ctypes.c_int), ("clip_norm", ctypes.c_float),
        ("seed", ctypes.c_uint64),
        ("gemm_mode", ctypes.c_int),
        ("channels", ctypes.c_int), ("image_size", ctypes.c_int), ("base_width", ctypes.c_int),
        ("t_embed", ctypes.c_int), ("timestep", ctypes.c_int),
        ("dense_targets", ctypes.c_int),
        ("embed_lr", ctypes.c_float),
    ]


GEMM_TF32, GEMM_FP32 = 0, 1


class Session:
    def __init__(self, **kw):
        self._lib = engine()
        d = SessionDesc()
        defaults = dict(lr=1e-3, adamw=1, clip_norm=1.0, fused_attention=1, key_grad_mode=KEYGRAD_REFERENCE,
                        seed=0)
        defaults.update(kw)
        for k, v in defaults.items():
            setattr(d, k, v)
        self.desc = d
        h = ctypes.c_void_p()
        self._lib.call("mle_session_create", ctypes.addressof(d), ctypes.addressof(h))
        self._h = h
        self.inputs = {}
        self.input_dev = {}
        name = ctypes.create_string_buffer(64)
        for i in range(self._lib.mle_session_input_count(h)):
            numel, dtype = ctypes.c_int64(), ctypes.c_int()
            hp, dp = ctypes.c_void_p(), ctypes.c_void_p()
            self._lib.call("mle_session_input_info", h, i, name, 64, ctypes.addressof(numel), ctypes.addressof(dtype),
                           ctypes.addressof(hp), ctypes.addressof(dp))
            ct = ctypes.c_float if dtype.value == 0 else ctypes.c_int32
            arr = np.ctypeslib.as_array((ct * numel.value).from_address(hp.value))
            self.inputs[name.value.decode()] = arr
            self.input_dev[name.value.decode()] = dp.value
        self.param_names = []
        self.param_sizes = []
        for i in range(self._lib.mle_session_param_count(h)):
            n = ctypes.c_int64()
            self._lib.call("mle_session_param_info", h, i, name, 64, ctypes.addressof(n))
            self.param_names.append(name.value.decode())
            self.param_sizes.append(n.value)

    # ------------------------------------------------------------ builders
    @classmethod
    def mlp(cls, batch=64, in_features=784, hidden=256, classes=10, **kw):
        # ReLU masks follow the pre-activation's sign: fp32 products keep
        # them identical to the reference's (the GEMMs here are tiny)
        kw.setdefault("gemm_mode", GEMM_FP32)
        return cls(config=MLP, batch=batch, in_features=in_features, hidden=hidden, classes=classes, **kw)

    @classmethod
    def encoder(cls, batch=32, seq_len=128, d_model=256, heads=8, ffn=1024, layers=2, vocab=4096, **kw):
        return cls(config=ENCODER, batch=batch, seq_len=seq_len, d_model=d_model, heads=heads, ffn=ffn,
                   layers=layers, vocab=vocab, **kw)

    @classmethod
    def encdec(cls, batch=256, seq_len=256, d_model=512, heads=8, ffn=2048, layers=6, vocab=8192, **kw):
        return cls(config=ENCDEC, batch=batch, seq_len=seq_len, d_model=d_model, heads=heads, ffn=ffn,
                   layers=layers, vocab=vocab, **kw)

    @classmethod
    def unet(cls, batch=32, channels=3, image_size=64, base_width=64, t_embed=256, timestep=500, **kw):
        """DDPM noise prediction; inputs "x_t" (noised images) and
        "noise" (the target), both [batch, channels, image_size, image_size]."""
        return cls(config=UNET, batch=batch, channels=channels, image_size=image_size, base_width=base_width,
                   t_embed=t_embed, timestep=timestep, **kw)

    # ---------------------------------------------------------------- step
    @property
    def stream(self):
        return self._lib.mle_session_stream(self._h)

    def step(self, upload=True, read_loss=True):
        loss = ctypes.c_float(float("nan"))
        self._lib.call("mle_session_step", self._h, int(upload), ctypes.addressof(loss) if read_loss else None)
        return loss.value if read_loss else None

    def phase(self, ph):
        self._lib.call("mle_session_phase", self._h, ph)

    def capture(self):
        self._lib.call("mle_session_capture", self._h)

    def capture_phases(self):
        """One CUDA graph per phase (0 zero_grad, 1 forward, 2 backward,
        3 gradient all-reduce, 4 clip, 5 update), device resident."""
        self._lib.call("mle_session_capture_phases", self._h)

    def phase_replay(self, ph):
        self._lib.call("mle_session_phase_replay", self._h, ph)

    def sync(self):
        self._lib.call("mle_session_sync", self._h)

    # ---------------------------------------------------------- parameters
    def read_param(self, i, which=0):
        out = np.empty(self.param_sizes[i], np.float32)
        self._lib.call("mle_session_param_read", self._h, i, which, out.ctypes.data)
        return out

    def write_param(self, i, data, which=0):
        data = np.ascontiguousarray(data, np.float32).ravel()
        if data.size != self.param_sizes[i]:
            raise MLEError(f"parameter {self.param_names[i]} has {self.param_sizes[i]} elements, got {data.size}")
        self._lib.call("mle_session_param_write", self._h, i, which, data.ctypes.data)

    def param_step(self, i):
        t = ctypes.c_int()
        self._lib.call("mle_session_param_step", self._h, i, ctypes.addressof(t))
        return t.value

    def save(self, path):
        """Checkpoint in the reference's AdamParameter::save record format
        (build order) plus `<path>.t` with the Adam steps."""
        self._lib.call("mle_session_save", self._h, str(path).encode())

    def load(self, path):
        self._lib.call("mle_session_load", self._h, str(path).encode())

    def write_embedding(self, i, table):
        table = np.ascontiguousarray(table, np.float32).ravel()
        self._lib.call("mle_session_embedding_write", self._h, i, table.ctypes.data, table.size)

    def read_embedding(self, i):
        n = self.desc.vocab * self.desc.d_model
        out = np.empty(n, np.float32)
        self._lib.call("mle_session_embedding_read", self._h, i, out.ctypes.data, n)
        return out

    def device_bytes(self):
        b = ctypes.c_int64()
        self._lib.call("mle_session_device_bytes", self._h, ctypes.addressof(b))
        return b.value

    def node_count(self):
        return self._lib.mle_session_node_count(self._h)

    def num_params(self):
        return int(sum(self.param_sizes))

    # ------------------------------------------------------------------- DP
    @staticmethod
    def dp_unique_id():
        buf = (ctypes.c_uint8 * 128)()
        engine().call("mle_dp_unique_id", ctypes.addressof(buf))
        return bytes(buf)

    def enable_dp(self, uid: bytes, rank: int, world: int, bucket_mb: int = 0):
        buf = (ctypes.c_uint8 * 128).from_buffer_copy(uid)
        self._lib.call("mle_session_enable_dp", self._h, ctypes.addressof(buf), rank, world, bucket_mb)

    def close(self):
        if self._h:
            self._lib.call("mle_session_destroy", self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
