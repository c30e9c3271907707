"""ctypes binding of libsa3k.so (include/sa3k.h) for tests, the benchmark and Python callers.

Device buffers are torch CUDA tensors (torch is only the allocator and stream here: every
computation runs in libsa3k's own kernels).  The library must have been built in-tree
(`python sa3.cpp_b200/build.py`); a missing library raises, there is no fallback.
"""
from __future__ import annotations

import ctypes
import weakref
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "lib", "libsa3k.so")

TYPE_IDS = {"f32": 0, "f16": 1, "q8_0": 8, "q4_k": 12}

# every symbol include/sa3k.h declares
ABI_SYMBOLS = (
    "sa3k_version", "sa3k_ctx_create", "sa3k_ctx_destroy", "sa3k_ctx_set_stream", "sa3k_sync", "sa3k_check_bounded_wait",
    "sa3k_weight_upload", "sa3k_weight_free", "sa3k_dequant", "sa3k_row_norms", "sa3k_col_norms", "sa3k_linear_fwd",
    "sa3k_linear_bwd", "sa3k_linear_fwd_bwd", "sa3k_linear_fwd_bwd_host", "sa3k_adamw",
    "sa3k_average_clip_adamw", "sa3k_profile_enable", "sa3k_profile_read", "sa3k_ctx_set_option",
    "sa3k_attention_fwd", "sa3k_attention_bwd", "sa3k_attention_bwd_noalloc", "sa3k_head_prep_fwd", "sa3k_head_prep_bwd",
    "sa3k_dit_create", "sa3k_dit_free", "sa3k_dit_set_tensor", "sa3k_dit_init_adapters", "sa3k_dit_adapter_size",
    "sa3k_dit_adapter_offsets", "sa3k_dit_adapter_buffer", "sa3k_dit_adapter_copy", "sa3k_dit_zero_grads",
    "sa3k_dit_forward_backward", "sa3k_dit_forward_backward_inpaint", "sa3k_dit_apply_adamw", "sa3k_dp_unique_id", "sa3k_dp_comm_create", "sa3k_dp_comm_create_timeout",
    "sa3k_dp_comm_destroy", "sa3k_dp_comm_info", "sa3k_dp_allreduce_sum", "sa3k_dp_allreduce_adamw",
    "sa3k_dit_dp_apply_adamw", "sa3k_dit_save_adapter", "sa3k_dit_load_adapter", "sa3k_dit_save_checkpoint",
    "sa3k_dit_load_checkpoint", "sa3k_adapter_gguf_write", "sa3k_gguf_get_string", "sa3k_gguf_get_u64",
    "sa3k_gguf_get_u64_array", "sa3k_gguf_get_f32", "sa3k_lora_chain_build", "sa3k_lora_chain_free",
    "sa3k_lora_chain_info", "sa3k_linear_fwd_chain", "sa3k_mat_effective_weight", "sa3k_linear_mat_fwd",
    "sa3k_linear_mat_fwd_bwd", "sa3k_dit_adapter_layout", "sa3k_dit_set_xs_bases",
)
OPT_WEIGHT_F16_CACHE, OPT_SMEM_DEQUANT, OPT_GEMM_TILE_N, OPT_GEMM_PAIR, OPT_ATTN_TC, OPT_PDL = 1, 2, 3, 4, 5, 6
OPT_STEP_GRAPH = 7
OPT_DEQUANT_TMEM = 8
OPT_FUSE_HEAD_PREP = 9


class Sa3kError(RuntimeError):
    pass


class Adapter(ctypes.Structure):
    _fields_ = [("A", ctypes.c_void_p), ("B", ctypes.c_void_p), ("magnitude", ctypes.c_void_p),
                ("base_norm_sq", ctypes.c_void_p), ("scale", ctypes.c_float), ("rank", ctypes.c_int)]


class Tensor4(ctypes.Structure):
    _fields_ = [("data", ctypes.c_void_p), ("batch_stride", ctypes.c_int64), ("head_stride", ctypes.c_int64),
                ("row_stride", ctypes.c_int64)]


class HeadSliceC(ctypes.Structure):
    _fields_ = [("col", ctypes.c_int), ("gamma", ctypes.c_void_p), ("rope", ctypes.c_int), ("rstd", ctypes.c_void_p)]


def t4(t, batch_stride, head_stride, row_stride):
    return Tensor4(ctypes.c_void_p(t.data_ptr()), batch_stride, head_stride, row_stride)


DIT_INT_FIELDS = ("io", "dim", "depth", "heads", "head_dim", "cond_dim", "mem_tokens", "rot", "time_dim",
                  "ff_inner", "differential")
DIT_FLOAT_FIELDS = ("rope_base", "norm_eps", "qk_eps", "time_min_freq", "time_max_freq")


class DitConfigC(ctypes.Structure):
    _fields_ = ([(n, ctypes.c_int) for n in DIT_INT_FIELDS] + [(n, ctypes.c_float) for n in DIT_FLOAT_FIELDS] +
                [("local_dim", ctypes.c_int)])


class ProfileEntry(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char * 48), ("launches", ctypes.c_int64), ("total_ms", ctypes.c_double)]


class ChainTerm(ctypes.Structure):
    """sa3k_chain_term: one adapter of an inference chain (device pointers)."""
    _fields_ = [("A", ctypes.c_void_p), ("B", ctypes.c_void_p), ("magnitude", ctypes.c_void_p), ("rank", ctypes.c_int),
                ("scale", ctypes.c_float)]


class MatAdapter(ctypes.Structure):
    """sa3k_mat_adapter: a materialized adapter of any family ("lora", "dora-rows", "dora-cols",
    "bora", each optionally "-xs"); every array a device pointer."""
    _fields_ = [("adapter_type", ctypes.c_char_p), ("rank", ctypes.c_int), ("scale", ctypes.c_float),
                ("A", ctypes.c_void_p), ("B", ctypes.c_void_p), ("U", ctypes.c_void_p), ("V", ctypes.c_void_p),
                ("M", ctypes.c_void_p), ("m", ctypes.c_void_p), ("m_r", ctypes.c_void_p), ("m_c", ctypes.c_void_p)]


class MatGrads(ctypes.Structure):
    """sa3k_mat_grads: the gradient outputs of sa3k_linear_mat_fwd_bwd (NULL where unused)."""
    _fields_ = [("dA", ctypes.c_void_p), ("dB", ctypes.c_void_p), ("dM", ctypes.c_void_p), ("dm", ctypes.c_void_p),
                ("dm_r", ctypes.c_void_p), ("dm_c", ctypes.c_void_p)]


def _vp(t):
    return None if t is None else t.data_ptr()


class TrainProgress(ctypes.Structure):
    """sa3k_train_progress: the dataset-side progress stored in a trainer-state file."""
    _fields_ = [("epoch", ctypes.c_uint64), ("next_sample", ctypes.c_uint64),
                ("order", ctypes.POINTER(ctypes.c_uint64)), ("n_order", ctypes.c_int64),
                ("compatibility", ctypes.c_char_p), ("rng_shuffle", ctypes.c_char_p), ("rng_crop", ctypes.c_char_p),
                ("rng_cfg", ctypes.c_char_p), ("rng_prompt", ctypes.c_char_p), ("rng_inpaint", ctypes.c_char_p),
                ("rng_diffusion", ctypes.c_char_p)]


class AdamWParams(ctypes.Structure):
    _fields_ = [("learning_rate", ctypes.c_float), ("beta1", ctypes.c_float), ("beta2", ctypes.c_float),
                ("eps", ctypes.c_float), ("weight_decay", ctypes.c_float), ("grad_clip", ctypes.c_float)]


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise Sa3kError(f"{LIB_PATH} is not built (python sa3.cpp_b200/build.py)")
        L = ctypes.CDLL(LIB_PATH)
        P, I, I64, F, E = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_float, ctypes.c_char_p
        L.sa3k_version.restype = ctypes.c_char_p
        L.sa3k_ctx_create.argtypes = [I, ctypes.POINTER(P), E, I]
        L.sa3k_ctx_destroy.argtypes = [P]
        L.sa3k_ctx_destroy.restype = None
        L.sa3k_ctx_set_stream.argtypes = [P, P, E, I]
        L.sa3k_sync.argtypes = [P, E, I]
        L.sa3k_check_bounded_wait.argtypes = [P, I, E, I]
        L.sa3k_weight_upload.argtypes = [P, I, P, I64, I64, ctypes.POINTER(P), E, I]
        L.sa3k_weight_free.argtypes = [P]
        L.sa3k_weight_free.restype = None
        L.sa3k_dequant.argtypes = [P, P, P, E, I]
        L.sa3k_row_norms.argtypes = [P, P, F, P, P, E, I]
        L.sa3k_linear_fwd.argtypes = [P, P, P, P, P, I64, P, E, I]
        L.sa3k_linear_bwd.argtypes = [P, P, P, P, P, P, P, I64, P, P, P, P, I, E, I]
        L.sa3k_linear_fwd_bwd.argtypes = [P, P, P, P, P, P, I64, P, P, P, P, P, E, I]
        L.sa3k_linear_fwd_bwd_host.argtypes = [P, P, P, P, P, P, I64, P, P, P, P, P, E, I]
        L.sa3k_adamw.argtypes = [P, P, P, P, P, I64, ctypes.POINTER(AdamWParams), I, E, I]
        L.sa3k_average_clip_adamw.argtypes = [P, P, P, P, P, I64, I, ctypes.POINTER(AdamWParams), I,
                                              ctypes.POINTER(ctypes.c_double), E, I]
        L.sa3k_profile_enable.argtypes = [P, I, E, I]
        L.sa3k_ctx_set_option.argtypes = [P, I, I64, E, I]
        L.sa3k_dit_create.argtypes = [P, ctypes.POINTER(DitConfigC), ctypes.POINTER(P), E, I]
        L.sa3k_dit_free.argtypes = [P]
        L.sa3k_dit_free.restype = None
        L.sa3k_dit_set_tensor.argtypes = [P, ctypes.c_char_p, I, P, I64, I64, E, I]
        L.sa3k_dit_init_adapters.argtypes = [P, ctypes.c_char_p, I, F, ctypes.POINTER(ctypes.c_char_p), I, E, I]
        L.sa3k_dit_adapter_size.argtypes = [P]
        L.sa3k_dit_adapter_offsets.argtypes = [P, I, ctypes.POINTER(I64), ctypes.POINTER(I64), ctypes.POINTER(I64)]
        L.sa3k_dit_adapter_buffer.argtypes = [P, I, ctypes.POINTER(P), E, I]
        L.sa3k_dit_adapter_layout.argtypes = [P, I, ctypes.POINTER(I64)]
        L.sa3k_dit_set_xs_bases.argtypes = [P, ctypes.c_char_p, P, P, E, I]
        L.sa3k_dit_adapter_copy.argtypes = [P, I, P, I64, I64, I, E, I]
        L.sa3k_dit_zero_grads.argtypes = [P, E, I]
        L.sa3k_dit_forward_backward.argtypes = [P, I, I, I, P, P, P, P, P, P, E, I]
        L.sa3k_dit_apply_adamw.argtypes = [P, I, ctypes.POINTER(AdamWParams), I, ctypes.POINTER(ctypes.c_double), E, I]
        T4 = ctypes.POINTER(Tensor4)
        L.sa3k_attention_fwd.argtypes = [P, I, I, I, I, I, F, I, T4, T4, T4, T4, P, E, I]
        L.sa3k_attention_bwd.argtypes = [P, I, I, I, I, I, F, I, T4, T4, T4, T4, T4, P, T4, T4, T4, E, I]
        L.sa3k_attention_bwd_noalloc.argtypes = [P, I, I, I, I, I, F, I, T4, T4, T4, T4, T4, P, T4, T4, T4, E, I]
        L.sa3k_head_prep_fwd.argtypes = [P, P, I, I, I, ctypes.POINTER(HeadSliceC), I, I, F, I, F, P, E, I]
        L.sa3k_head_prep_bwd.argtypes = [P, P, I64, P, I, I, I, ctypes.POINTER(HeadSliceC), I, I, F, P, E, I]
        L.sa3k_dp_unique_id.argtypes = [P, I, E, I]
        L.sa3k_dp_comm_create.argtypes = [P, I, I, P, ctypes.POINTER(P), E, I]
        L.sa3k_dp_comm_create_timeout.argtypes = [P, I, I, P, ctypes.c_double, ctypes.POINTER(P), E, I]
        L.sa3k_dp_comm_destroy.argtypes = [P]
        L.sa3k_dp_comm_destroy.restype = None
        L.sa3k_dp_comm_info.argtypes = [P, ctypes.POINTER(I), ctypes.POINTER(I)]
        L.sa3k_dp_allreduce_sum.argtypes = [P, P, P, I64, E, I]
        L.sa3k_dp_allreduce_adamw.argtypes = [P, P, P, P, P, P, I64, I, ctypes.POINTER(AdamWParams), I,
                                              ctypes.POINTER(ctypes.c_double), E, I]
        L.sa3k_dit_dp_apply_adamw.argtypes = [P, P, I, ctypes.POINTER(AdamWParams), I,
                                              ctypes.POINTER(ctypes.c_double), E, I]
        L.sa3k_profile_read.argtypes = [P, ctypes.POINTER(ProfileEntry), I, ctypes.POINTER(I), E, I]
        L.sa3k_lora_chain_build.argtypes = [P, P, ctypes.POINTER(ChainTerm), I, ctypes.POINTER(P), E, I]
        L.sa3k_lora_chain_free.argtypes = [P]
        L.sa3k_lora_chain_free.restype = None
        L.sa3k_lora_chain_info.argtypes = [P, ctypes.POINTER(I), ctypes.POINTER(I)]
        L.sa3k_linear_fwd_chain.argtypes = [P, P, P, P, P, I64, P, E, I]
        L.sa3k_mat_effective_weight.argtypes = [P, P, ctypes.POINTER(MatAdapter), P, E, I]
        L.sa3k_linear_mat_fwd.argtypes = [P, P, ctypes.POINTER(MatAdapter), P, P, I64, P, E, I]
        L.sa3k_linear_mat_fwd_bwd.argtypes = [P, P, ctypes.POINTER(MatAdapter), P, P, P, I64, P, P,
                                              ctypes.POINTER(MatGrads), E, I]
        L.sa3k_dit_save_adapter.argtypes = [P, E, E, I]
        L.sa3k_dit_load_adapter.argtypes = [P, E, E, I]
        L.sa3k_dit_save_checkpoint.argtypes = [P, E, E, I64, ctypes.POINTER(TrainProgress), E, I]
        L.sa3k_dit_load_checkpoint.argtypes = [P, E, E, ctypes.POINTER(I64), E, I]
        PP = ctypes.POINTER(ctypes.c_void_p)
        L.sa3k_adapter_gguf_write.argtypes = [E, E, I, F, I, ctypes.POINTER(ctypes.c_char_p), ctypes.POINTER(I64),
                                              ctypes.POINTER(I64), PP, PP, PP, E, I]
        L.sa3k_gguf_get_string.argtypes = [E, E, E, I64, ctypes.POINTER(I64), E, I]
        L.sa3k_gguf_get_u64.argtypes = [E, E, ctypes.POINTER(ctypes.c_uint64), E, I]
        L.sa3k_gguf_get_u64_array.argtypes = [E, E, ctypes.POINTER(ctypes.c_uint64), I64, ctypes.POINTER(I64), E, I]
        L.sa3k_gguf_get_f32.argtypes = [E, E, P, I64, ctypes.POINTER(I64), ctypes.POINTER(I64), ctypes.POINTER(I), E, I]
        for name in ABI_SYMBOLS:
            if name not in ("sa3k_version", "sa3k_ctx_destroy", "sa3k_weight_free", "sa3k_dit_free",
                            "sa3k_dp_comm_destroy", "sa3k_lora_chain_free"):
                getattr(L, name).restype = I
        L.sa3k_dit_adapter_size.restype = I64
        _lib = L
    return _lib


def _ptr(t):
    if t is None:
        return None
    if hasattr(t, "data_ptr"):
        return ctypes.c_void_p(t.data_ptr())
    if hasattr(t, "ctypes"):
        return t.ctypes.data_as(ctypes.c_void_p)
    return t


def _check(rc, err):
    if rc != 0:
        raise Sa3kError(err.value.decode(errors="replace"))


class Context:
    """A sa3k context bound to one CUDA device (and, by default, torch's current stream)."""

    def __init__(self, device=0, use_torch_stream=True):
        self._h = ctypes.c_void_p()
        err = ctypes.create_string_buffer(512)
        _check(lib().sa3k_ctx_create(device, ctypes.byref(self._h), err, 512), err)
        self.device = device
        if use_torch_stream:
            import torch
            s = torch.cuda.current_stream(device).cuda_stream
            self.set_stream(s)

    def set_stream(self, stream_handle):
        err = ctypes.create_string_buffer(256)
        _check(lib().sa3k_ctx_set_stream(self._h, ctypes.c_void_p(stream_handle), err, 256), err)

    def set_option(self, option, value):
        err = ctypes.create_string_buffer(256)
        _check(lib().sa3k_ctx_set_option(self._h, option, int(value), err, 256), err)

    def sync(self):
        err = ctypes.create_string_buffer(512)
        _check(lib().sa3k_sync(self._h, err, 512), err)

    def check_bounded_wait(self, limit_us):
        """Launch the bounded-wait probe (a wait that runs out after limit_us); the next sync()
        raises with the timeout."""
        err = ctypes.create_string_buffer(512)
        _check(lib().sa3k_check_bounded_wait(self._h, int(limit_us), err, 512), err)

    def _own(self, obj):
        """Objects made on this context (weights, models, communicators) are released before it."""
        if not hasattr(self, "_children"):
            self._children = weakref.WeakSet()
        self._children.add(obj)

    def close(self):
        for obj in list(getattr(self, "_children", ())):
            obj.close()
        if self._h:
            lib().sa3k_ctx_destroy(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def profile_enable(self, timing=1):
        """timing 0: count launches only; 1: time each launch class with events (eager);
        2: events captured into a CUDA graph, re-read after each replay."""
        err = ctypes.create_string_buffer(256)
        _check(lib().sa3k_profile_enable(self._h, int(timing), err, 256), err)

    def profile_read(self):
        """{class name: (launches, total_ms)} since the last profile_enable."""
        err = ctypes.create_string_buffer(256)
        n = ctypes.c_int(0)
        _check(lib().sa3k_profile_read(self._h, None, 0, ctypes.byref(n), err, 256), err)
        arr = (ProfileEntry * max(n.value, 1))()
        _check(lib().sa3k_profile_read(self._h, arr, n.value, ctypes.byref(n), err, 256), err)
        return {arr[i].name.decode(): (arr[i].launches, arr[i].total_ms) for i in range(n.value)}

    # -------------------------------------------------------------------- attention
    def attention_fwd(self, B, H, Sq, Sk, scale, window, q, k, v, o, lse):
        err = ctypes.create_string_buffer(512)
        _check(lib().sa3k_attention_fwd(self._h, B, H, Sq, Sk, 64, scale, window, ctypes.byref(q), ctypes.byref(k),
                                        ctypes.byref(v), ctypes.byref(o), _ptr(lse), err, 512), err)

    def attention_bwd(self, B, H, Sq, Sk, scale, window, q, k, v, o, dO, lse, dq, dk=None, dv=None):
        err = ctypes.create_string_buffer(512)
        _check(lib().sa3k_attention_bwd(self._h, B, H, Sq, Sk, 64, scale, window, ctypes.byref(q), ctypes.byref(k),
                                        ctypes.byref(v), ctypes.byref(o), ctypes.byref(dO), _ptr(lse), ctypes.byref(dq),
                                        ctypes.byref(dk) if dk else None, ctypes.byref(dv) if dv else None, err, 512),
               err)

    def attention_bwd_noalloc(self, B, H, Sq, Sk, scale, window, q, k, v, o, dO, lse, dq, dk=None, dv=None):
        """attention_bwd with its scratch in a fixed library array (B*H*Sq <= 2**20); see sa3k.h."""
        err = ctypes.create_string_buffer(512)
        _check(lib().sa3k_attention_bwd_noalloc(self._h, B, H, Sq, Sk, 64, scale, window, ctypes.byref(q),
                                                ctypes.byref(k), ctypes.byref(v), ctypes.byref(o), ctypes.byref(dO),
                                                _ptr(lse), ctypes.byref(dq), ctypes.byref(dk) if dk else None,
                                                ctypes.byref(dv) if dv else None, err, 512), err)

    def head_prep_fwd(self, y, T, ncols, H, slices, tps, eps, rot, base, out):
        err = ctypes.create_string_buffer(512)
        arr = (HeadSliceC * len(slices))(*slices)
        _check(lib().sa3k_head_prep_fwd(self._h, _ptr(y), T, ncols, H, arr, len(slices), tps, eps, rot, base, _ptr(out),
                                        err, 512), err)

    def head_prep_bwd(self, g, g_ld, y, T, ncols, H, sl, tps, rot, base, dy):
        err = ctypes.create_string_buffer(512)
        _check(lib().sa3k_head_prep_bwd(self._h, _ptr(g), g_ld, _ptr(y), T, ncols, H, ctypes.byref(sl), tps, rot, base,
                                        _ptr(dy), err, 512), err)

    # -------------------------------------------------------------------- weights
    def upload(self, raw_bytes, qtype, inn, out):
        import numpy as np
        raw = np.ascontiguousarray(raw_bytes)
        h = ctypes.c_void_p()
        err = ctypes.create_string_buffer(512)
        _check(lib().sa3k_weight_upload(self._h, TYPE_IDS[qtype], raw.ctypes.data_as(ctypes.c_void_p),
                                        inn, out, ctypes.byref(h), err, 512), err)
        return Weight(self, h, qtype, inn, out)

    # -------------------------------------------------------------------- ops
    def dequant(self, w, dst):
        err = ctypes.create_string_buffer(512)
        _check(lib().sa3k_dequant(self._h, w._h, _ptr(dst), err, 512), err)

    def row_norms(self, w, eps, nsq=None, nrm=None):
        err = ctypes.create_string_buffer(512)
        _check(lib().sa3k_row_norms(self._h, w._h, eps, _ptr(nsq), _ptr(nrm), err, 512), err)

    @staticmethod
    def adapter(A, B, scale, m=None, bns=None):
        rank = A.shape[0]
        return Adapter(_ptr(A), _ptr(B), _ptr(m), _ptr(bns), scale, rank)

    def linear_fwd(self, w, x, y, ad=None, bias=None):
        err = ctypes.create_string_buffer(512)
        _check(lib().sa3k_linear_fwd(self._h, w._h, ctypes.byref(ad) if ad else None, _ptr(bias), _ptr(x),
                                     x.shape[0], _ptr(y), err, 512), err)

    def lora_chain(self, w, terms):
        """terms: list of (A [rank][in], B [out][rank], magnitude [out] or None, scale) torch cuda f32 tensors,
        in chain order.  Returns a LoraChain (folded on the device)."""
        arr = (ChainTerm * len(terms))(*[ChainTerm(A.data_ptr(), B.data_ptr(), m.data_ptr() if m is not None else None,
                                                   A.shape[0], s) for A, B, m, s in terms])
        h = ctypes.c_void_p()
        err = ctypes.create_string_buffer(512)
        _check(lib().sa3k_lora_chain_build(self._h, w._h, arr, len(terms), ctypes.byref(h), err, 512), err)
        return LoraChain(h)

    def linear_fwd_chain(self, w, chain, x, y, bias=None):
        err = ctypes.create_string_buffer(512)
        _check(lib().sa3k_linear_fwd_chain(self._h, w._h, chain._h, _ptr(bias), _ptr(x), x.shape[0], _ptr(y), err,
                                           512), err)

    @staticmethod
    def mat_adapter(adapter_type, rank, scale, A=None, B=None, U=None, V=None, M=None, m=None, m_r=None, m_c=None):
        """A MatAdapter over device tensors (kept alive by the caller)."""
        return MatAdapter(adapter_type.encode(), rank, scale, _vp(A), _vp(B), _vp(U), _vp(V), _vp(M), _vp(m), _vp(m_r),
                          _vp(m_c))

    def mat_effective_weight(self, w, ad, weff):
        err = ctypes.create_string_buffer(512)
        _check(lib().sa3k_mat_effective_weight(self._h, w._h, ctypes.byref(ad), _ptr(weff), err, 512), err)

    def linear_mat_fwd(self, w, ad, x, y, bias=None):
        err = ctypes.create_string_buffer(512)
        _check(lib().sa3k_linear_mat_fwd(self._h, w._h, ctypes.byref(ad), _ptr(bias), _ptr(x), x.shape[0], _ptr(y),
                                         err, 512), err)

    def linear_mat_fwd_bwd(self, w, ad, x, dy, y=None, dx=None, bias=None, dA=None, dB=None, dM=None, dm=None,
                           dm_r=None, dm_c=None):
        err = ctypes.create_string_buffer(512)
        g = MatGrads(_vp(dA), _vp(dB), _vp(dM), _vp(dm), _vp(dm_r), _vp(dm_c))
        _check(lib().sa3k_linear_mat_fwd_bwd(self._h, w._h, ctypes.byref(ad), _ptr(bias), _ptr(x), _ptr(dy),
                                             x.shape[0], _ptr(y), _ptr(dx), ctypes.byref(g), err, 512), err)

    def linear_bwd(self, w, x, y, dy, dx, ad=None, bias=None, dA=None, dB=None, dm=None, accumulate=False):
        err = ctypes.create_string_buffer(512)
        _check(lib().sa3k_linear_bwd(self._h, w._h, ctypes.byref(ad) if ad else None, _ptr(bias), _ptr(x),
                                     _ptr(y), _ptr(dy), x.shape[0], _ptr(dx), _ptr(dA), _ptr(dB), _ptr(dm),
                                     1 if accumulate else 0, err, 512), err)

    def linear_fwd_bwd(self, w, x, dy, y, dx, ad=None, bias=None, dA=None, dB=None, dm=None):
        err = ctypes.create_string_buffer(512)
        _check(lib().sa3k_linear_fwd_bwd(self._h, w._h, ctypes.byref(ad) if ad else None, _ptr(bias), _ptr(x),
                                         _ptr(dy), x.shape[0], _ptr(y), _ptr(dx), _ptr(dA), _ptr(dB), _ptr(dm),
                                         err, 512), err)

    def linear_fwd_bwd_host(self, w, x, dy, y, dx, ad=None, bias=None, dA=None, dB=None, dm=None):
        """All arguments are numpy float32 arrays (host memory); ad holds host pointers."""
        err = ctypes.create_string_buffer(512)
        _check(lib().sa3k_linear_fwd_bwd_host(self._h, w._h, ctypes.byref(ad) if ad else None, _ptr(bias),
                                              _ptr(x), _ptr(dy), x.shape[0], _ptr(y), _ptr(dx), _ptr(dA),
                                              _ptr(dB), _ptr(dm), err, 512), err)

    def adamw(self, p, g, m, v, hp: AdamWParams, step):
        err = ctypes.create_string_buffer(512)
        _check(lib().sa3k_adamw(self._h, _ptr(p), _ptr(g), _ptr(m), _ptr(v), p.numel(), ctypes.byref(hp),
                                step, err, 512), err)

    def average_clip_adamw(self, p, g, m, v, count, hp: AdamWParams, step, want_norm=False):
        err = ctypes.create_string_buffer(512)
        norm = ctypes.c_double(0.0)
        _check(lib().sa3k_average_clip_adamw(self._h, _ptr(p), _ptr(g), _ptr(m), _ptr(v), p.numel(), count,
                                             ctypes.byref(hp), step, ctypes.byref(norm) if want_norm else None,
                                             err, 512), err)
        return norm.value if want_norm else None


class Weight:
    def __init__(self, ctx, h, qtype, inn, out):
        self.ctx, self._h, self.qtype, self.inn, self.out = ctx, h, qtype, inn, out
        ctx._own(self)

    def free(self):
        if self._h:
            lib().sa3k_weight_free(self._h)
            self._h = ctypes.c_void_p()

    close = free

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


class LoraChain:
    def __init__(self, h):
        self._h = h

    def info(self):
        r, f = ctypes.c_int(), ctypes.c_int()
        lib().sa3k_lora_chain_info(self._h, ctypes.byref(r), ctypes.byref(f))
        return r.value, bool(f.value)

    def free(self):
        if self._h:
            lib().sa3k_lora_chain_free(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


class Dit:
    """A DiT training model on a context (sa3k_dit_*): tensors by GGUF name, flat adapter state."""

    def __init__(self, ctx, cfg):
        self.ctx = ctx
        c = DitConfigC(**{k: cfg[k] for k in DIT_INT_FIELDS + DIT_FLOAT_FIELDS}, local_dim=cfg.get("local_dim", 0))
        self._h = ctypes.c_void_p()
        err = ctypes.create_string_buffer(512)
        _check(lib().sa3k_dit_create(ctx._h, ctypes.byref(c), ctypes.byref(self._h), err, 512), err)
        ctx._own(self)

    def close(self):
        if self._h:
            lib().sa3k_dit_free(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def set_tensor(self, name, qtype, host, ne0, ne1=1):
        import numpy as np
        a = np.ascontiguousarray(host)
        if qtype == "f32" and a.nbytes < 4 * ne0 * max(ne1, 1):
            raise Sa3kError(f"{name}: host buffer holds {a.nbytes} bytes, [{ne1}][{ne0}] f32 needs more")
        err = ctypes.create_string_buffer(512)
        _check(lib().sa3k_dit_set_tensor(self._h, name.encode(), TYPE_IDS[qtype], a.ctypes.data_as(ctypes.c_void_p),
                                         ne0, ne1, err, 512), err)

    def init_adapters(self, adapter_type, rank, alpha, names):
        arr = (ctypes.c_char_p * len(names))(*[n.encode() for n in names])
        err = ctypes.create_string_buffer(512)
        _check(lib().sa3k_dit_init_adapters(self._h, adapter_type.encode(), rank, alpha, arr, len(names), err, 512), err)

    def size(self):
        return int(lib().sa3k_dit_adapter_size(self._h))

    def offsets(self, idx):
        a, b, m = ctypes.c_int64(), ctypes.c_int64(), ctypes.c_int64()
        if lib().sa3k_dit_adapter_offsets(self._h, idx, ctypes.byref(a), ctypes.byref(b), ctypes.byref(m)):
            raise Sa3kError("bad target index")
        return a.value, b.value, m.value

    def layout(self, idx):
        """(A, B, row magnitude, column magnitude, M_xs) offsets of target idx, -1 where absent."""
        offs = (ctypes.c_int64 * 5)()
        if lib().sa3k_dit_adapter_layout(self._h, idx, offs):
            raise Sa3kError("bad target index")
        return tuple(int(v) for v in offs)

    def set_xs_bases(self, name, U, V):
        import numpy as np
        U = np.ascontiguousarray(U, np.float32)
        V = np.ascontiguousarray(V, np.float32)
        err = ctypes.create_string_buffer(512)
        _check(lib().sa3k_dit_set_xs_bases(self._h, name.encode(), _ptr(U), _ptr(V), err, 512), err)

    def copy(self, which, buf, offset=0, count=None, to_model=True):
        """which: 0 params, 1 grads, 2 AdamW m, 3 AdamW v; buf: numpy float32 (host) or torch tensor."""
        n = count if count is not None else (buf.size if hasattr(buf, "size") and not callable(buf.size) else buf.numel())
        err = ctypes.create_string_buffer(512)
        _check(lib().sa3k_dit_adapter_copy(self._h, which, _ptr(buf), offset, n, 1 if to_model else 0, err, 512), err)

    def buffer_ptr(self, which):
        p = ctypes.c_void_p()
        err = ctypes.create_string_buffer(256)
        _check(lib().sa3k_dit_adapter_buffer(self._h, which, ctypes.byref(p), err, 256), err)
        return p.value

    def save_adapter(self, path):
        """The adapters as the reference's adapter GGUF (loads in its generator)."""
        err = ctypes.create_string_buffer(512)
        _check(lib().sa3k_dit_save_adapter(self._h, path.encode(), err, 512), err)

    def load_adapter(self, path):
        err = ctypes.create_string_buffer(512)
        _check(lib().sa3k_dit_load_adapter(self._h, path.encode(), err, 512), err)

    def save_checkpoint(self, adapter_path, state_path, step, epoch=0, next_sample=0, order=(0,), compatibility="",
                        rng=None):
        """Immutable adapter + trainer-state pair; rng: dict of the sampler states (shuffle, crop, cfg, prompt,
        inpaint, diffusion) as strings."""
        rng = rng or {}
        order_arr = (ctypes.c_uint64 * len(order))(*order)
        pr = TrainProgress(epoch, next_sample, order_arr, len(order), compatibility.encode(),
                           *[rng.get(k, "").encode() for k in ("shuffle", "crop", "cfg", "prompt", "inpaint",
                                                               "diffusion")])
        err = ctypes.create_string_buffer(512)
        _check(lib().sa3k_dit_save_checkpoint(self._h, adapter_path.encode(), state_path.encode(), step,
                                              ctypes.byref(pr), err, 512), err)

    def load_checkpoint(self, adapter_path, state_path):
        """Restores parameters and AdamW moments; returns the step (the rest of the progress is read with
        gguf_get_*)."""
        err = ctypes.create_string_buffer(512)
        st = ctypes.c_int64()
        _check(lib().sa3k_dit_load_checkpoint(self._h, adapter_path.encode(), state_path.encode(), ctypes.byref(st),
                                              err, 512), err)
        return st.value

    def zero_grads(self):
        err = ctypes.create_string_buffer(256)
        _check(lib().sa3k_dit_zero_grads(self._h, err, 256), err)

    def forward_backward(self, B, T, ctx_len, x_t, target, t_feat, cross, glob, loss=None):
        err = ctypes.create_string_buffer(1024)
        _check(lib().sa3k_dit_forward_backward(self._h, B, T, ctx_len, _ptr(x_t), _ptr(target), _ptr(t_feat),
                                               _ptr(cross), _ptr(glob), _ptr(loss), err, 1024), err)

    def forward_backward_inpaint(self, B, T, ctx_len, x_t, target, t_feat, cross, glob, local, loss_weight, loss=None):
        """forward_backward with the inpaint local conditioning [B][T][local_dim] and loss weights [B][T][io]."""
        err = ctypes.create_string_buffer(1024)
        _check(lib().sa3k_dit_forward_backward_inpaint(self._h, B, T, ctx_len, _ptr(x_t), _ptr(target), _ptr(t_feat),
                                                       _ptr(cross), _ptr(glob), _ptr(local), _ptr(loss_weight),
                                                       _ptr(loss), err, 1024), err)

    def dp_apply_adamw(self, comm, samples_per_rank, hp, step, want_norm=False):
        """All-reduce the gradients over comm's ranks, then AdamW with count = samples_per_rank x ranks."""
        err = ctypes.create_string_buffer(512)
        norm = ctypes.c_double(0.0)
        _check(lib().sa3k_dit_dp_apply_adamw(self._h, comm._h, samples_per_rank, ctypes.byref(hp), step,
                                             ctypes.byref(norm) if want_norm else None, err, 512), err)
        return norm.value if want_norm else None

    def apply_adamw(self, count, hp, step, want_norm=False):
        err = ctypes.create_string_buffer(512)
        norm = ctypes.c_double(0.0)
        _check(lib().sa3k_dit_apply_adamw(self._h, count, ctypes.byref(hp), step,
                                          ctypes.byref(norm) if want_norm else None, err, 512), err)
        return norm.value if want_norm else None


# ------------------------------------------------------------------------ data parallel
def dp_unique_id():
    """128 bytes identifying a new NCCL clique (make on one rank, hand to all)."""
    buf = ctypes.create_string_buffer(128)
    err = ctypes.create_string_buffer(512)
    _check(lib().sa3k_dp_unique_id(buf, 128, err, 512), err)
    return buf.raw


class DpComm:
    """A data-parallel communicator of nranks processes, one per GPU (sa3k_dp_comm_*)."""

    def __init__(self, ctx, nranks, rank, unique_id, timeout_s=None):
        """timeout_s: bound on the rendezvous (every rank must join within it; default 300 s)."""
        assert len(unique_id) == 128
        self.ctx = ctx
        self._h = ctypes.c_void_p()
        uid = ctypes.create_string_buffer(bytes(unique_id), 128)
        err = ctypes.create_string_buffer(512)
        if timeout_s is None:
            _check(lib().sa3k_dp_comm_create(ctx._h, nranks, rank, uid, ctypes.byref(self._h), err, 512), err)
        else:
            _check(lib().sa3k_dp_comm_create_timeout(ctx._h, nranks, rank, uid, float(timeout_s),
                                                     ctypes.byref(self._h), err, 512), err)
        self.nranks, self.rank = nranks, rank
        ctx._own(self)

    def allreduce_sum(self, buf, n=None):
        n = buf.numel() if n is None else n
        err = ctypes.create_string_buffer(512)
        _check(lib().sa3k_dp_allreduce_sum(self.ctx._h, self._h, _ptr(buf), n, err, 512), err)

    def allreduce_adamw(self, p, g, m, v, samples_per_rank, hp, step, want_norm=False):
        err = ctypes.create_string_buffer(512)
        norm = ctypes.c_double(0.0)
        _check(lib().sa3k_dp_allreduce_adamw(self.ctx._h, self._h, _ptr(p), _ptr(g), _ptr(m), _ptr(v), p.numel(),
                                             samples_per_rank, ctypes.byref(hp), step,
                                             ctypes.byref(norm) if want_norm else None, err, 512), err)
        return norm.value if want_norm else None

    def close(self):
        if self._h:
            lib().sa3k_dp_comm_destroy(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


# ------------------------------------------------------------------ GGUF adapter / trainer-state files
def adapter_gguf_write(path, adapter_type, rank, alpha, targets):
    """targets: list of (stem, A [rank][in], B [out][rank], m [out] or None), numpy float32."""
    import numpy as np
    n = len(targets)
    arrs = [(np.ascontiguousarray(A, np.float32), np.ascontiguousarray(Bm, np.float32),
             None if m is None else np.ascontiguousarray(m, np.float32)) for _, A, Bm, m in targets]
    stems = (ctypes.c_char_p * n)(*[t[0].encode() for t in targets])
    ins = (ctypes.c_int64 * n)(*[a[0].shape[1] for a in arrs])
    outs = (ctypes.c_int64 * n)(*[a[1].shape[0] for a in arrs])
    Ap = (ctypes.c_void_p * n)(*[a[0].ctypes.data for a in arrs])
    Bp = (ctypes.c_void_p * n)(*[a[1].ctypes.data for a in arrs])
    Mp = (ctypes.c_void_p * n)(*[(a[2].ctypes.data if a[2] is not None else None) for a in arrs])
    err = ctypes.create_string_buffer(512)
    _check(lib().sa3k_adapter_gguf_write(path.encode(), adapter_type.encode(), rank, alpha, n, stems, ins, outs, Ap,
                                         Bp, Mp, err, 512), err)


def gguf_get_string(path, key):
    err = ctypes.create_string_buffer(512)
    n = ctypes.c_int64()
    _check(lib().sa3k_gguf_get_string(path.encode(), key.encode(), None, 0, ctypes.byref(n), err, 512), err)
    buf = ctypes.create_string_buffer(n.value + 1)
    _check(lib().sa3k_gguf_get_string(path.encode(), key.encode(), buf, n.value + 1, None, err, 512), err)
    return buf.raw[:n.value].decode()


def gguf_get_u64(path, key):
    err = ctypes.create_string_buffer(512)
    v = ctypes.c_uint64()
    _check(lib().sa3k_gguf_get_u64(path.encode(), key.encode(), ctypes.byref(v), err, 512), err)
    return v.value


def gguf_get_u64_array(path, key):
    err = ctypes.create_string_buffer(512)
    n = ctypes.c_int64()
    _check(lib().sa3k_gguf_get_u64_array(path.encode(), key.encode(), None, 0, ctypes.byref(n), err, 512), err)
    out = (ctypes.c_uint64 * max(n.value, 1))()
    _check(lib().sa3k_gguf_get_u64_array(path.encode(), key.encode(), out, n.value, ctypes.byref(n), err, 512), err)
    return list(out[:n.value])


def gguf_get_f32(path, name):
    """(values as a flat numpy float32 array, ne tuple with ne[0] innermost)."""
    import numpy as np
    err = ctypes.create_string_buffer(512)
    n = ctypes.c_int64()
    ne = (ctypes.c_int64 * 4)()
    nd = ctypes.c_int()
    _check(lib().sa3k_gguf_get_f32(path.encode(), name.encode(), None, 0, ctypes.byref(n), ne, ctypes.byref(nd), err,
                                   512), err)
    out = np.empty(n.value, np.float32)
    _check(lib().sa3k_gguf_get_f32(path.encode(), name.encode(), out.ctypes.data_as(ctypes.c_void_p), n.value,
                                   ctypes.byref(n), ne, ctypes.byref(nd), err, 512), err)
    return out, tuple(ne[:nd.value])
