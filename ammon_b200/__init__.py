"""ammon_b200: B200-native Ammon decode layer path.

Python host mirror of the Ammon crate's public API over the C ABI
(include/ammon_b200.h): ``create_runtime`` (src/gpu.rs), ``Scheme`` (Goldy's
record-then-replay scheme), ``DecodeStep`` (src/kernels.rs:10-33), ``Tensor``, the
kernels of src/kernels.rs (``kernels``), the modules of src/modules.rs
(``Embedding``, ``RmsNorm``, ``Linear``, ``CausalAttentionBlock``, ``SwiGluBlock``,
``KvCache``), the host loop (``generate_tokens``, ``sample_argmax``,
``AutoregressiveModel``) and a Llama-shaped model assembly (``LlamaModel``).

All compute runs in libammon_b200.so (sm_100a CUDA kernels). There is no CPU
fallback: without the library, or without a GPU, calls raise.
"""
from __future__ import annotations

import ctypes as C
import os
from dataclasses import dataclass
from typing import Iterable, List, Optional, Sequence

import numpy as np

from . import _abi
from ._abi import AB_BF16, AB_F32, AB_U32
from .generate import (AutoregressiveModel, GenerateOptions, GenerateOutput,
                       GenerateTokenOutput, generate, generate_tokens)
from .tokenizer import BpeTokenizer, NativeBpeTokenizer, Tokenizer, sample_argmax

DEFAULT_ROPE_THETA = 10000.0  # src/kernels.rs:8
ATTENTION_SPLIT = 8           # src/kernels.rs:229
ATTENTION_MAX_HEAD = 128      # src/kernels.rs:231

F32, BF16, U32 = AB_F32, AB_BF16, AB_U32
_NP = {AB_F32: np.float32, AB_BF16: np.uint16, AB_U32: np.uint32}


class AmmonError(RuntimeError):
    def __init__(self, code, message):
        super().__init__(message)
        self.code = code


class ValidationError(AmmonError):
    """A shape / dtype contract violation (GoldyError::Validation)."""


class DeviceError(AmmonError):
    """A kernel flagged an out-of-range token or position."""


def load():
    return _abi.lib()


def _check(status):
    if status != _abi.AB_OK:
        msg = (_abi.lib().ab_last_error() or b"").decode(errors="replace")
        cls = {_abi.AB_ERR_VALIDATION: ValidationError,
               _abi.AB_ERR_DEVICE: DeviceError}.get(status, AmmonError)
        raise cls(status, msg)


# --------------------------------------------------------------------------- runtime
class Runtime:
    """CUDA device + stream (src/gpu.rs create_runtime)."""

    def __init__(self, device: int = 0):
        h = C.c_void_p()
        _check(_abi.lib().ab_runtime_create(device, C.byref(h)))
        self._h = h
        self.device = device

    @property
    def handle(self):
        return self._h

    def synchronize(self):
        _check(_abi.lib().ab_runtime_synchronize(self._h))

    @property
    def stream(self) -> int:
        return int(_abi.lib().ab_runtime_stream(self._h) or 0)

    @property
    def sm_count(self) -> int:
        n = C.c_int32()
        _check(_abi.lib().ab_runtime_sm_count(self._h, C.byref(n)))
        return n.value

    @property
    def wait_limit_ms(self) -> int:
        """Limit of every bounded wait in this runtime's kernels (milliseconds)."""
        n = C.c_uint32()
        _check(_abi.lib().ab_runtime_wait_limit(self._h, C.byref(n)))
        return n.value

    @wait_limit_ms.setter
    def wait_limit_ms(self, ms: int):
        _check(_abi.lib().ab_runtime_set_wait_limit(self._h, int(ms)))

    def scheme(self) -> "Scheme":
        return Scheme(self)

    def deposit(self, parcel: "Tensor", steps: Sequence["DecodeStep"]):
        arr = (_abi.DecodeStep_t * len(steps))(*[(s.token, s.position) for s in steps])
        _check(_abi.lib().ab_step_deposit(self._h, parcel.t, arr, len(steps)))

    def close(self):
        if getattr(self, "_h", None):
            _abi.lib().ab_runtime_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def create_runtime(device: int = 0) -> Runtime:
    return Runtime(device)


# --------------------------------------------------------------------------- tensors
class Tensor:
    """Contiguous row-major device tensor view (goldy::Tensor / TensorView)."""

    def __init__(self, t: _abi.Tensor_t, rt: Optional[Runtime] = None, owner=None,
                 owned: bool = False):
        self.t = t
        self.rt = rt
        self._owner = owner  # keeps the memory alive (a parent Tensor or a torch tensor)
        self._owned = owned

    # construction -------------------------------------------------------------
    @staticmethod
    def _desc(ptr, dtype, shape) -> _abi.Tensor_t:
        shape = tuple(int(s) for s in shape)
        if not 1 <= len(shape) <= 4:
            raise ValueError("rank must be 1..4")
        d = _abi.Tensor_t()
        d.data = ptr
        d.dtype = dtype
        d.rank = len(shape)
        for i, s in enumerate(shape):
            d.dims[i] = s
        return d

    @classmethod
    def zeros(cls, rt: Runtime, shape, dtype=AB_F32) -> "Tensor":
        shape = tuple(int(s) for s in shape)
        dims = (C.c_uint32 * len(shape))(*shape)
        t = _abi.Tensor_t()
        _check(_abi.lib().ab_tensor_zeros(rt.handle, dtype, len(shape), dims, C.byref(t)))
        return cls(t, rt, owned=True)

    @classmethod
    def from_array(cls, rt: Runtime, arr, dtype=None, shape=None) -> "Tensor":
        arr = np.asarray(arr)
        if dtype is None:
            dtype = AB_BF16 if arr.dtype == np.uint16 else (AB_U32 if arr.dtype == np.uint32
                                                           else AB_F32)
        arr = np.ascontiguousarray(arr, dtype=_NP[dtype])
        t = cls.zeros(rt, shape if shape is not None else (arr.shape or (1,)), dtype)
        t.write(arr)
        return t

    @classmethod
    def from_f32(cls, rt: Runtime, shape, values) -> "Tensor":
        return cls.from_array(rt, np.asarray(values, np.float32).reshape(shape), AB_F32)

    @classmethod
    def from_torch(cls, tensor, rt: Optional[Runtime] = None) -> "Tensor":
        import torch

        if not tensor.is_contiguous():
            raise ValueError("tensor must be contiguous")
        dt = {torch.float32: AB_F32, torch.bfloat16: AB_BF16, torch.int32: AB_U32,
              torch.uint32: AB_U32}[tensor.dtype]
        return cls(cls._desc(tensor.data_ptr(), dt, tuple(tensor.shape) or (1,)), rt,
                   owner=tensor)

    # views ---------------------------------------------------------------------
    @property
    def shape(self):
        return tuple(self.t.dims[i] for i in range(self.t.rank))

    @property
    def dtype(self):
        return self.t.dtype

    @property
    def numel(self):
        return int(np.prod(self.shape))

    @property
    def nbytes(self):
        return self.numel * (2 if self.dtype == AB_BF16 else 4)

    @property
    def data_ptr(self):
        return int(self.t.data or 0)

    def narrow(self, dim, start, length) -> "Tensor":
        if dim != 0:
            raise ValueError("narrow is supported on dim 0 (contiguous views)")
        out = _abi.Tensor_t()
        _check(_abi.lib().ab_tensor_narrow(self.t, start, length, C.byref(out)))
        return Tensor(out, self.rt, owner=self)

    def reshape(self, shape) -> "Tensor":
        shape = tuple(int(s) for s in shape)
        dims = (C.c_uint32 * len(shape))(*shape)
        out = _abi.Tensor_t()
        _check(_abi.lib().ab_tensor_reshape(self.t, len(shape), dims, C.byref(out)))
        return Tensor(out, self.rt, owner=self)

    def view(self) -> "Tensor":
        return self

    # data -----------------------------------------------------------------------
    def write(self, arr):
        arr = np.ascontiguousarray(arr, dtype=_NP[self.dtype])
        _check(_abi.lib().ab_tensor_write(self.rt.handle, self.t, arr.ctypes.data, arr.nbytes))

    def read(self) -> np.ndarray:
        """Waits for the runtime stream and returns a host copy (uint16 bits for bf16)."""
        out = np.empty(self.shape, _NP[self.dtype])
        _check(_abi.lib().ab_tensor_read(self.rt.handle, self.t, out.ctypes.data, out.nbytes))
        return out

    def read_f32(self) -> np.ndarray:
        a = self.read()
        if self.dtype == AB_BF16:
            return (a.astype(np.uint32) << 16).view(np.float32)
        return a

    def fill_normal(self, seed, stream, mean=0.0, std=1.0):
        _check(_abi.lib().ab_tensor_fill_normal(self.rt.handle, self.t, seed, stream, mean, std))
        return self

    def free(self):
        if self._owned and self.t.data:
            _abi.lib().ab_tensor_free(self.rt.handle, C.byref(self.t))
            self._owned = False

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


@dataclass
class DecodeStep:
    """Token and sequence position uploaded each decode step (src/kernels.rs:10-15)."""
    token: int = 0
    position: int = 0

    @staticmethod
    def parcel(rt: Runtime, n: int = 1) -> Tensor:
        """Retained device parcel of n steps (src/kernels.rs:17-27)."""
        t = _abi.Tensor_t()
        _check(_abi.lib().ab_step_parcel(rt.handle, n, C.byref(t)))
        return Tensor(t, rt, owned=True)


# --------------------------------------------------------------------------- schemes
class Scheme:
    """Recorded dispatch list replayed as one CUDA graph (goldy::Scheme)."""

    def __init__(self, rt: Optional[Runtime]):
        h = C.c_void_p()
        _check(_abi.lib().ab_scheme_create(rt.handle if rt else None, C.byref(h)))
        self._h = h
        self.rt = rt
        self._keep: List[object] = []

    @property
    def handle(self):
        return self._h

    def submit(self) -> "Scheme":
        _check(_abi.lib().ab_scheme_submit(self._h))
        return self

    def ir_node_count(self) -> int:
        n = C.c_uint32()
        _check(_abi.lib().ab_scheme_node_count(self._h, C.byref(n)))
        return n.value

    def replay_stats(self):
        r, p = C.c_uint32(), C.c_uint32()
        _check(_abi.lib().ab_scheme_replay_stats(self._h, C.byref(r), C.byref(p)))
        return ReplayStats(records=r.value, replays=p.value)

    def use_graph(self, enable: bool):
        _check(_abi.lib().ab_scheme_use_graph(self._h, 1 if enable else 0))

    def node_labels(self) -> List[str]:
        out = []
        buf = C.create_string_buffer(128)
        for i in range(self.ir_node_count()):
            _check(_abi.lib().ab_scheme_node_label(self._h, i, buf, 128))
            out.append(buf.value.decode())
        return out

    def time_nodes(self, iters: int = 10) -> List[float]:
        """Mean milliseconds per launch of each node, each launched on its own between CUDA
        events on the runtime stream."""
        n = self.ir_node_count()
        arr = (C.c_float * max(n, 1))()
        _check(_abi.lib().ab_scheme_time_nodes(self._h, iters, arr, max(n, 1)))
        return [float(arr[i]) for i in range(n)]

    def keep(self, *objs):
        self._keep.extend(objs)

    def close(self):
        if getattr(self, "_h", None):
            _abi.lib().ab_scheme_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


@dataclass
class ReplayStats:
    records: int
    replays: int
    specialization_promotions: int = 0


# --------------------------------------------------------------------------- modules
def _t(x: Tensor):
    return x.t


class Embedding:
    """Token embedding table gather (src/modules.rs:100-132)."""

    def __init__(self, rt: Runtime):
        self.rt = rt

    def record(self, scheme: Scheme, table: Tensor, step: Tensor, x: Tensor):
        _check(_abi.lib().ab_embedding_record(scheme.handle, table.t, step.t, x.t))
        scheme.keep(table, step, x)


class RmsNorm:
    """RMSNorm (src/modules.rs:135-164)."""

    def __init__(self, rt: Runtime):
        self.rt = rt

    def record(self, scheme: Scheme, x: Tensor, weight: Tensor, out: Tensor):
        _check(_abi.lib().ab_rmsnorm_record(scheme.handle, x.t, weight.t, out.t))
        scheme.keep(x, weight, out)

    def record_inplace(self, scheme: Scheme, x: Tensor, weight: Tensor):
        _check(_abi.lib().ab_rmsnorm_record_inplace(scheme.handle, x.t, weight.t))
        scheme.keep(x, weight)


class Linear:
    """Dense projection out = weight @ x (src/modules.rs:167-187)."""

    def __init__(self, rt: Runtime):
        self.rt = rt

    def record(self, scheme: Scheme, weight: Tensor, x: Tensor, out: Tensor):
        _check(_abi.lib().ab_linear_record(scheme.handle, weight.t, x.t, out.t))
        scheme.keep(weight, x, out)


@dataclass
class KvLayer:
    key: Tensor
    value: Tensor


class KvCache:
    """Persistent key/value cache [layers, (batch,) seq, kv_heads, head] (src/modules.rs:38-64)."""

    def __init__(self, rt: Runtime, layers, seq_len, kv_heads, head_size, dtype=AB_F32,
                 batch=1):
        h = C.c_void_p()
        _check(_abi.lib().ab_kvcache_create(rt.handle, layers, seq_len, kv_heads, head_size,
                                            dtype, batch, C.byref(h)))
        self._h = h
        self.rt = rt

    @classmethod
    def _borrow(cls, rt, handle):
        obj = cls.__new__(cls)
        obj._h = handle
        obj.rt = rt
        obj._borrowed = True
        return obj

    def layer(self, layer: int) -> KvLayer:
        k, v = _abi.Tensor_t(), _abi.Tensor_t()
        _check(_abi.lib().ab_kvcache_layer(self._h, layer, C.byref(k), C.byref(v)))
        return KvLayer(Tensor(k, self.rt, owner=self), Tensor(v, self.rt, owner=self))

    def zero(self):
        _check(_abi.lib().ab_kvcache_zero(self._h))

    def close(self):
        if getattr(self, "_h", None) and not getattr(self, "_borrowed", False):
            _abi.lib().ab_kvcache_destroy(self._h)
        self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


@dataclass
class CausalAttentionBlockWeights:
    norm: Tensor
    query: Tensor
    key: Tensor
    value: Tensor
    output: Tensor


@dataclass
class SwiGluBlockWeights:
    norm: Tensor
    gate: Tensor
    up: Tensor
    down: Tensor


class CausalAttentionBlock:
    """Pre-norm causal attention block (src/modules.rs:192-274)."""

    def __init__(self, rt: Runtime, hidden, query_heads, seq_len, max_batch=1,
                 rope_theta=DEFAULT_ROPE_THETA):
        h = C.c_void_p()
        _check(_abi.lib().ab_attention_block_create(rt.handle, hidden, query_heads, seq_len,
                                                    max_batch, rope_theta, C.byref(h)))
        self._h = h
        self.rt = rt

    def record(self, scheme: Scheme, x: Tensor, weights: CausalAttentionBlockWeights,
               cache: KvLayer, step: Tensor):
        w = _abi.AttentionWeights_t(weights.norm.t, weights.query.t, weights.key.t,
                                    weights.value.t, weights.output.t)
        _check(_abi.lib().ab_attention_block_record(self._h, scheme.handle, x.t, C.byref(w),
                                                    cache.key.t, cache.value.t, step.t))
        scheme.keep(self, x, weights, cache, step)

    def close(self):
        if getattr(self, "_h", None):
            _abi.lib().ab_attention_block_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class SwiGluBlock:
    """Pre-norm SwiGLU block (src/modules.rs:279-333)."""

    def __init__(self, rt: Runtime, hidden, intermediate, max_batch=1):
        h = C.c_void_p()
        _check(_abi.lib().ab_swiglu_block_create(rt.handle, hidden, intermediate, max_batch,
                                                 C.byref(h)))
        self._h = h
        self.rt = rt

    def record(self, scheme: Scheme, x: Tensor, weights: SwiGluBlockWeights):
        w = _abi.SwigluWeights_t(weights.norm.t, weights.gate.t, weights.up.t, weights.down.t)
        _check(_abi.lib().ab_swiglu_block_record(self._h, scheme.handle, x.t, C.byref(w)))
        scheme.keep(self, x, weights)

    def close(self):
        if getattr(self, "_h", None):
            _abi.lib().ab_swiglu_block_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


# --------------------------------------------------------------------------- model
WEIGHT_IDS = {"embed": 0, "wcls": 1, "rms_final": 2, "rms_att": 3, "wq": 4, "wk": 5, "wv": 6,
              "wo": 7, "rms_ffn": 8, "w1": 9, "w2": 10, "w3": 11}


@dataclass
class LlamaConfig:
    dim: int
    layers: int
    heads: int
    kv_heads: int
    head_dim: int
    hidden: int
    vocab: int
    seq: int
    batch: int = 1
    rope_theta: float = DEFAULT_ROPE_THETA
    norm_eps: float = 1e-5
    dtype: int = AB_F32

    def weight_bytes(self) -> int:
        qd, kvd = self.heads * self.head_dim, self.kv_heads * self.head_dim
        per_layer = 2 * qd * self.dim + 2 * kvd * self.dim + 3 * self.hidden * self.dim
        elems = self.layers * per_layer + 2 * self.vocab * self.dim
        return elems * (2 if self.dtype == AB_BF16 else 4)


class Comm:
    """NCCL communicator of one rank (tensor parallelism over NVLink). Rank 0 makes the id
    with ``Comm.unique_id()`` and shares it with the other ranks (e.g. a torch.distributed
    broadcast); every rank then builds its Comm with the same id."""

    def __init__(self, rt: Runtime, uid: bytes, rank: int, world: int,
                 timeout_ms: Optional[int] = None):
        if len(uid) != _abi.COMM_ID_BYTES:
            raise ValueError("communicator id must be 128 bytes")
        buf = (C.c_uint8 * _abi.COMM_ID_BYTES).from_buffer_copy(uid)
        h = C.c_void_p()
        if timeout_ms is None:
            _check(_abi.lib().ab_comm_create(rt.handle, buf, rank, world, C.byref(h)))
        else:
            _check(_abi.lib().ab_comm_create_timeout(rt.handle, buf, rank, world,
                                                     int(timeout_ms), C.byref(h)))
        self._h = h
        self.rt = rt
        self.rank, self.world = rank, world

    @staticmethod
    def unique_id() -> bytes:
        buf = (C.c_uint8 * _abi.COMM_ID_BYTES)()
        _check(_abi.lib().ab_comm_unique_id(buf))
        return bytes(buf)

    @staticmethod
    def loopback_reduce(rt: Runtime, world: int, ready: int, n: int) -> np.ndarray:
        """ab_comm_loopback_reduce: the all-reduce kernel over `world` ranks held in this
        GPU's memory, ranks outside the `ready` mask never arriving."""
        out = np.zeros(n, np.float32)
        _check(_abi.lib().ab_comm_loopback_reduce(
            rt.handle, world, ready, n, out.ctypes.data_as(C.POINTER(C.c_float))))
        return out

    @property
    def handle(self):
        return self._h

    def abort(self):
        if getattr(self, "_h", None):
            _abi.lib().ab_comm_abort(self._h)

    def close(self):
        if getattr(self, "_h", None):
            _abi.lib().ab_comm_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class LlamaModel:
    """Llama-shaped decode model on the fused kernels (an architecture-crate role the
    reference leaves open, README.md:5,21). ``step`` is AutoregressiveModel::step.
    With ``comm`` the model is this rank's tensor-parallel shard."""

    def __init__(self, rt: Runtime, cfg: LlamaConfig, comm: Optional[Comm] = None):
        c = _abi.LlamaConfig_t(cfg.dim, cfg.layers, cfg.heads, cfg.kv_heads, cfg.head_dim,
                               cfg.hidden, cfg.vocab, cfg.seq, cfg.batch, cfg.rope_theta,
                               cfg.norm_eps, cfg.dtype)
        h = C.c_void_p()
        if comm is None:
            _check(_abi.lib().ab_llama_create(rt.handle, C.byref(c), C.byref(h)))
        else:
            _check(_abi.lib().ab_llama_create_tp(rt.handle, C.byref(c), comm.handle,
                                                 C.byref(h)))
        self._h = h
        self.rt = rt
        self.cfg = cfg
        self.comm = comm
        self._logits = np.zeros((cfg.batch, cfg.vocab), np.float32)
        self._argmax = np.zeros(cfg.batch, np.int32)
        self._register_logits()

    def _register_logits(self):
        """Page-locks the logits buffer so step() fills it straight from the device."""
        self._registered = _abi.lib().ab_host_register(
            self._logits.ctypes.data, self._logits.nbytes) == _abi.AB_OK

    @classmethod
    def from_llama2c(cls, rt: Runtime, path: str, dtype: int = AB_F32, batch: int = 1,
                     rope_theta: float = DEFAULT_ROPE_THETA,
                     comm: Optional[Comm] = None) -> "LlamaModel":
        """A model with the weights of a llama2.c checkpoint (run.c layout; the reference
        leaves checkpoints to architecture crates, README.md:5,21). With ``comm`` every rank
        loads its own shard from the same file."""
        c = _abi.LlamaConfig_t()
        h = C.c_void_p()
        _check(_abi.lib().ab_llama_load_llama2c(
            rt.handle, os.fsencode(path), dtype, batch, rope_theta,
            comm.handle if comm is not None else None, C.byref(c), C.byref(h)))
        self = cls.__new__(cls)
        self._h = h
        self.rt = rt
        self.cfg = LlamaConfig(c.dim, c.layers, c.heads, c.kv_heads, c.head_dim, c.hidden,
                               c.vocab, c.seq, c.batch, c.rope_theta, c.norm_eps, c.dtype)
        self.comm = comm
        self._logits = np.zeros((c.batch, c.vocab), np.float32)
        self._argmax = np.zeros(c.batch, np.int32)
        self._register_logits()
        return self

    @staticmethod
    def llama2c_config(path: str, batch: int = 1, dtype: int = AB_F32,
                       rope_theta: float = DEFAULT_ROPE_THETA) -> "LlamaConfig":
        """The model shape a llama2.c checkpoint holds (header and file size checked; no
        GPU needed)."""
        c = _abi.LlamaConfig_t()
        _check(_abi.lib().ab_llama2c_config(os.fsencode(path), batch, dtype, rope_theta,
                                            C.byref(c)))
        return LlamaConfig(c.dim, c.layers, c.heads, c.kv_heads, c.head_dim, c.hidden,
                           c.vocab, c.seq, c.batch, c.rope_theta, c.norm_eps, c.dtype)

    @property
    def handle(self):
        return self._h

    def init_synthetic(self, seed: int, std: float = 0.02):
        _check(_abi.lib().ab_llama_init_synthetic(self._h, seed, std))

    def weight(self, name: str, layer: int = 0) -> Tensor:
        t = _abi.Tensor_t()
        _check(_abi.lib().ab_llama_weight(self._h, WEIGHT_IDS[name], layer, C.byref(t)))
        return Tensor(t, self.rt, owner=self)

    def cache(self) -> KvCache:
        h = C.c_void_p()
        _check(_abi.lib().ab_llama_cache(self._h, C.byref(h)))
        return KvCache._borrow(self.rt, h)

    def reset(self):
        _check(_abi.lib().ab_llama_reset(self._h))

    def vocab_size(self) -> int:
        return self.cfg.vocab

    def max_seq_len(self) -> int:
        return self.cfg.seq

    def step_batch(self, tokens: Sequence[int], positions: Sequence[int], logits=True,
                   argmax=False):
        n = self.cfg.batch
        arr = (_abi.DecodeStep_t * n)(*[(int(t), int(p)) for t, p in zip(tokens, positions)])
        lp = self._logits.ctypes.data_as(C.POINTER(C.c_float)) if logits else None
        ap = self._argmax.ctypes.data_as(C.POINTER(C.c_int32)) if argmax else None
        _check(_abi.lib().ab_llama_step(self._h, arr, n, lp, ap))
        return (self._logits if logits else None), (self._argmax if argmax else None)

    def step(self, token: int, pos: int) -> np.ndarray:
        """AutoregressiveModel::step (src/model.rs:10): host logits of one token."""
        logits, _ = self.step_batch([token], [pos])
        return logits[0]

    def prefill(self, tokens: Sequence[int], pos0: int = 0, stream: int = 0,
                logits: bool = True):
        """Runs prompt `tokens` of cache stream `stream` at positions pos0.. as batched
        passes (each weight read once per pass); returns (last token's logits or None, its
        greedy id). The cache ends as one step per token leaves it (src/generate.rs:60-66)."""
        toks = np.ascontiguousarray(tokens, np.int32)
        out = np.zeros(self.cfg.vocab, np.float32) if logits else None
        am = C.c_int32()
        _check(_abi.lib().ab_llama_prefill(
            self._h, int(stream), toks.ctypes.data_as(C.POINTER(C.c_int32)), toks.size,
            int(pos0), out.ctypes.data_as(C.POINTER(C.c_float)) if logits else None,
            C.byref(am)))
        return out, int(am.value)

    def prefill_scheme(self, rows: int, stream: int = 0, head: bool = True) -> "Scheme":
        """The recorded prefill pass of `rows` positions (profiling; owned by the model)."""
        h = C.c_void_p()
        _check(_abi.lib().ab_llama_prefill_scheme(self._h, int(stream), int(rows),
                                                  1 if head else 0, C.byref(h)))
        s = Scheme.__new__(Scheme)
        s._h = h
        s.rt = self.rt
        s._keep = [self]
        s.close = lambda: None
        return s

    def prefill_launches(self) -> int:
        """Graph nodes (kernels and collectives) the last prefill launched."""
        n = C.c_uint32()
        _check(_abi.lib().ab_llama_prefill_launches(self._h, C.byref(n)))
        return int(n.value)

    def set_prefill_rows(self, rows: int):
        """Rows per prefill pass (1..256; 0 = the default 256)."""
        _check(_abi.lib().ab_llama_prefill_rows(self._h, int(rows)))

    def generate(self, prompt: Sequence[int], max_new_tokens: int,
                 stop_on: Optional[int] = None) -> GenerateTokenOutput:
        """generate_tokens (src/generate.rs:43-91) with the prompt prefilled in batched passes
        and each new token picked by the device argmax (batch-1 model)."""
        prompt = np.ascontiguousarray(prompt, np.int32)
        cap = max(int(max_new_tokens), 1)
        out = np.zeros(cap, np.int32)
        n = C.c_uint32()
        tps = C.c_double()
        _check(_abi.lib().ab_llama_generate_tokens(
            self._h, prompt.ctypes.data_as(C.POINTER(C.c_int32)), prompt.size,
            int(max_new_tokens), 0 if stop_on is None else 1,
            0 if stop_on is None else int(stop_on), out.ctypes.data_as(C.POINTER(C.c_int32)),
            cap, C.byref(n), C.byref(tps)))
        return GenerateTokenOutput(tokens=out[:min(n.value, cap)].tolist(),
                                   prompt_tokens=int(prompt.size),
                                   tokens_per_second=float(tps.value))

    def decode_device(self, tokens: Sequence[int], positions: Sequence[int], steps: int,
                      want_tokens: bool = True):
        """Greedy decode of `steps` tokens entirely on the device, starting from one
        DecodeStep per batch row. Returns [steps, batch] ids (or None)."""
        n = self.cfg.batch
        arr = (_abi.DecodeStep_t * n)(*[(int(t), int(p)) for t, p in zip(tokens, positions)])
        out = np.zeros((steps, n), np.int32) if want_tokens else None
        _check(_abi.lib().ab_llama_decode_device(
            self._h, arr, n, steps,
            out.ctypes.data_as(C.POINTER(C.c_int32)) if want_tokens else None))
        return out

    def scheme(self) -> "Scheme":
        h = C.c_void_p()
        _check(_abi.lib().ab_llama_scheme(self._h, C.byref(h)))
        s = Scheme.__new__(Scheme)
        s._h = h
        s.rt = self.rt
        s._keep = [self]
        s.close = lambda: None  # owned by the model
        return s

    def step_trace(self):
        """[barriers, 4, grid] %globaltimer ns of each CTA at each grid barrier of the last
        persistent decode step (arrival, release, operand staged, partial rows pushed at an
        all-reduce site; AMMON_B200_STEP_TRACE set at creation), or None."""
        nb, ng = C.c_uint32(), C.c_uint32()
        _check(_abi.lib().ab_llama_step_trace(self._h, None, 0, C.byref(nb), C.byref(ng)))
        if nb.value == 0:
            return None
        out = np.zeros((nb.value, 4, ng.value), np.uint64)
        _check(_abi.lib().ab_llama_step_trace(
            self._h, out.ctypes.data_as(C.POINTER(C.c_uint64)), out.size, C.byref(nb),
            C.byref(ng)))
        return out

    def logits_tensor(self) -> Tensor:
        t = _abi.Tensor_t()
        _check(_abi.lib().ab_llama_logits(self._h, C.byref(t)))
        return Tensor(t, self.rt, owner=self)

    def generate_tokens_native(self, prompt: Sequence[int], max_new_tokens: int,
                               stop_on: Optional[int] = None) -> GenerateTokenOutput:
        """generate_tokens (src/generate.rs:43-91) run by the C++ host loop."""
        vt = _abi.Model_t()
        _check(_abi.lib().ab_llama_as_model(self._h, C.byref(vt)))
        return _native_generate(vt, prompt, max_new_tokens, stop_on)

    def close(self):
        if getattr(self, "_h", None):
            _abi.lib().ab_llama_destroy(self._h)
            self._h = None
        if getattr(self, "_registered", False):
            _abi.lib().ab_host_unregister(self._logits.ctypes.data)
            self._registered = False

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def _native_generate(vt, prompt, max_new_tokens, stop_on) -> GenerateTokenOutput:
    prompt = np.ascontiguousarray(prompt, np.int32)
    cap = max(int(max_new_tokens), 1)
    out = np.zeros(cap, np.int32)
    n = C.c_uint32()
    tps = C.c_double()
    _check(_abi.lib().ab_generate_tokens(
        C.byref(vt), prompt.ctypes.data_as(C.POINTER(C.c_int32)), prompt.size,
        int(max_new_tokens), 0 if stop_on is None else 1,
        0 if stop_on is None else int(stop_on), out.ctypes.data_as(C.POINTER(C.c_int32)), cap,
        C.byref(n), C.byref(tps)))
    return GenerateTokenOutput(tokens=out[:min(n.value, cap)].tolist(),
                               prompt_tokens=int(prompt.size),
                               tokens_per_second=float(tps.value))


def native_generate_tokens(model, prompt, max_new_tokens, stop_on=None) -> GenerateTokenOutput:
    """Runs the C++ generate_tokens over any Python AutoregressiveModel (through ctypes
    callbacks). Used to test the native loop's semantics without a GPU."""
    keep = {}

    def _vocab(_):
        return int(model.vocab_size())

    def _seq(_):
        return int(model.max_seq_len())

    def _step(_, token, pos, out):
        try:
            logits = np.ascontiguousarray(model.step(int(token), int(pos)), np.float32)
        except Exception:
            return _abi.AB_ERR_ARGUMENT
        keep["l"] = logits
        out[0] = logits.ctypes.data_as(C.POINTER(C.c_float))
        return _abi.AB_OK

    vt = _abi.Model_t(None, _abi.VOCAB_FN(_vocab), _abi.SEQ_FN(_seq), _abi.STEP_FN(_step))
    keep["vt"] = vt
    return _native_generate(vt, prompt, max_new_tokens, stop_on)


def native_sample_argmax(logits) -> int:
    a = np.ascontiguousarray(logits, np.float32)
    return int(_abi.lib().ab_sample_argmax(a.ctypes.data_as(C.POINTER(C.c_float)), a.size))


from . import kernels  # noqa: E402  (the reference's kernel-level API)

__all__ = [
    "AmmonError", "ValidationError", "DeviceError", "Runtime", "create_runtime", "Tensor",
    "DecodeStep", "Scheme", "Embedding", "RmsNorm", "Linear", "KvCache", "KvLayer",
    "CausalAttentionBlock", "CausalAttentionBlockWeights", "SwiGluBlock",
    "SwiGluBlockWeights", "LlamaConfig", "LlamaModel", "Comm", "AutoregressiveModel",
    "generate_tokens", "generate", "GenerateOptions", "GenerateOutput", "GenerateTokenOutput",
    "sample_argmax", "BpeTokenizer", "NativeBpeTokenizer", "Tokenizer", "kernels",
    "DEFAULT_ROPE_THETA",
    "ATTENTION_SPLIT", "ATTENTION_MAX_HEAD", "F32", "BF16", "U32", "load",
]
