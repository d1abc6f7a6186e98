"""The reference's kernel-level API (src/kernels.rs): ``XKernel.prepare(runtime)``
then ``.record(scheme, label, ...)``.

Launch geometry is chosen by the library, so the returned dispatch accepts the
reference's ``over_1d`` / ``over_tensor`` / ``groups`` calls as no-ops.
"""
from __future__ import annotations

from . import _abi

DEFAULT_ROPE_THETA = 10000.0
ATTENTION_SPLIT = 8
ATTENTION_MAX_HEAD = 128


class Dispatch:
    def over_1d(self, n):
        return self

    def over_tensor(self, t):
        return self

    def groups(self, g):
        return self


class _Kernel:
    fn = None

    def __init__(self, rt=None):
        self.rt = rt

    @classmethod
    def prepare(cls, rt):
        return cls(rt)

    def _rec(self, scheme, *tensors, extra=()):
        from . import _check

        _check(getattr(_abi.lib(), self.fn)(scheme.handle, *[t.t for t in tensors], *extra))
        scheme.keep(*tensors)
        return Dispatch()


class EmbedKernel(_Kernel):
    fn = "ab_kernel_embed"

    def record(self, scheme, label, embed, step, x):
        return self._rec(scheme, embed, step, x)


class GemvKernel(_Kernel):
    fn = "ab_kernel_gemv"

    def record(self, scheme, label, x, w, xout, step):
        return self._rec(scheme, x, w, xout, step)


class RmsnormKernel(_Kernel):
    fn = "ab_kernel_rmsnorm"

    def record(self, scheme, label, x, weight, o):
        return self._rec(scheme, x, weight, o)


class RmsnormInplaceKernel(_Kernel):
    fn = "ab_kernel_rmsnorm_inplace"

    def record(self, scheme, label, x, weight):
        return self._rec(scheme, x, weight)


class RopeKernel(_Kernel):
    fn = "ab_kernel_rope"

    def record(self, scheme, label, q, k, step, theta):
        return self._rec(scheme, q, k, step, extra=(float(theta),))


class RopeStoreKernel(_Kernel):
    fn = "ab_kernel_rope_store"

    def record(self, scheme, label, q, k_proj, k, step, theta):
        return self._rec(scheme, q, k_proj, k, step, extra=(float(theta),))


class CacheStoreKernel(_Kernel):
    fn = "ab_kernel_cache_store"

    def record(self, scheme, label, src, dst, step):
        return self._rec(scheme, src, dst, step)


class AttentionPartialKernel(_Kernel):
    fn = "ab_kernel_attention_partial"

    def record(self, scheme, label, q, key_cache, value_cache, partial, step):
        return self._rec(scheme, q, key_cache, value_cache, partial, step)


class AttentionCombineKernel(_Kernel):
    fn = "ab_kernel_attention_combine"

    def record(self, scheme, label, partial, xb, step):
        return self._rec(scheme, partial, xb, step)


class AttentionDecodeKernel(_Kernel):
    """The fused flash-decoding replacement of AttentionPartialKernel + AttentionCombineKernel
    (src/kernels.rs:228-410): one recorded kernel, split scratch owned by the scheme. q is
    [heads, head] or [batch, heads, head]; the caches gain a leading batch dim with it."""

    fn = "ab_kernel_attention_decode"

    def record(self, scheme, label, q, key_cache, value_cache, out, step):
        return self._rec(scheme, q, key_cache, value_cache, out, step)


class AttentionKernel(_Kernel):
    fn = "ab_kernel_attention"

    def record(self, scheme, label, q, att, xb, key_cache, value_cache, step):
        return self._rec(scheme, q, att, xb, key_cache, value_cache, step)


class SwigluKernel(_Kernel):
    fn = "ab_kernel_swiglu"

    def record(self, scheme, label, hb, hb2):
        return self._rec(scheme, hb, hb2)


class TensorKernels(_Kernel):
    """Residual add and matmul (src/kernels.rs:495-534)."""

    def add_into(self, scheme, label, a, b, out):
        self.fn = "ab_tensor_add_into"
        return self._rec(scheme, a, b, out)

    def matmul_into(self, scheme, label, a, b, out):
        self.fn = "ab_tensor_matmul_into"
        return self._rec(scheme, a, b, out)
