"""ctypes binding of libqw6cuda.so (the in-tree CUDA library).

Two layers, mirroring the C headers in include/:

* qw6_vk.h -- the drop-in per-call entry points of qw6's Vulkan backend
  (host memory in and out, synchronous, 0 / -1).  Exposed as functions with
  the same names minus the ``qw6_vk_`` prefix; -1 raises Qw6CudaError.
* qw6_cuda.h -- the device-resident API (``Context``): device pointers (ints,
  e.g. ``torch.Tensor.data_ptr()``), work enqueued on the context's stream.

There is no CPU fallback: if the shared library is missing or no B200 is
usable, the calls raise.
"""
from __future__ import annotations

import ctypes as C
import subprocess
from pathlib import Path

import numpy as np

PKG = Path(__file__).resolve().parent
LIB_PATH = PKG / "libqw6cuda.so"
CSRC = PKG / "csrc"

# qw6_quant_t (qw6.h:77-92)
Q4_K, Q4_K_S, Q5_K, Q6_K, IQ3_S, IQ2_S, IQ2_XXS = 4, 5, 6, 7, 9, 11, 13
FP32 = 0
BLOCK_BYTES = {Q4_K: 144, Q4_K_S: 144, Q5_K: 176, Q6_K: 210, IQ2_XXS: 66, IQ2_S: 82, IQ3_S: 110}

# Symbols include/*.h declare (checked by tests/test_abi.py).
VK_SYMBOLS = (
    "qw6_vk_selftest", "qw6_vk_matvec_f32_host", "qw6_vk_matmul_q4k_host", "qw6_vk_matmul_q5k_host",
    "qw6_vk_matmul_q6k_host", "qw6_vk_matmul_iq2xxs_host", "qw6_vk_matmul_iq2s_host",
    "qw6_vk_matmul_iq3s_host", "qw6_vk_silu_mul_host", "qw6_vk_argmax_host", "qw6_vk_sampling_greedy_host",
    "qw6_vk_moe_route_host", "qw6_vk_moe_gather_host", "qw6_vk_rmsnorm_host", "qw6_vk_rmsnorm_chunked_host",
    "qw6_vk_attention_gqa_host", "qw6_vk_deltanet_conv1d_host", "qw6_vk_deltanet_retrieve_host",
    "qw6_vk_deltanet_update_host", "qw6_vk_mrope_host", "qw6_vk_mtp_draft_host", "qw6_vk_pipe_init",
    "qw6_vk_pipe_forward", "qw6_vk_pipe_forward_greedy", "qw6_vk_pipe_free",
)


class Qw6CudaError(RuntimeError):
    pass


class GgufTensor(C.Structure):
    _fields_ = [("name", C.c_char_p), ("n_dims", C.c_uint32), ("dims", C.c_uint64 * 4), ("ggml_type", C.c_uint32),
                ("quant", C.c_int), ("file_offset", C.c_uint64), ("bytes", C.c_uint64), ("data", C.c_void_p)]


class MoeTable(C.Structure):
    _fields_ = [("n_layers", C.c_uint32), ("packs", C.c_void_p), ("packs_dev", C.c_void_p), ("weights", C.c_void_p),
                ("bytes", C.c_size_t)]


def build(jobs: int = 8) -> None:
    """Compile libqw6cuda.so in-tree (sm_100a)."""
    subprocess.run(["make", "-s", f"-j{jobs}", "-C", str(CSRC)], check=True)


_lib = None

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C")
_u32p = np.ctypeslib.ndpointer(np.uint32, flags="C")
_u8p = np.ctypeslib.ndpointer(np.uint8, flags="C")
_vp = C.c_void_p
_u32 = C.c_uint32
_sz = C.c_size_t


class ModelTensor(C.Structure):
    """qw6cu_model_tensor: one host tensor of a model for the decoder."""
    _fields_ = [("field", C.c_uint32), ("layer", C.c_int32), ("quant", C.c_uint32), ("rows", C.c_uint32),
                ("cols", C.c_uint32), ("data", C.c_void_p), ("stride", C.c_size_t)]


class ExpertPack(C.Structure):
    _fields_ = [("quant", C.c_uint32), ("base", C.c_void_p), ("stride", C.c_size_t)]


class SharedExpert(C.Structure):
    """qw6cu_shared_expert: gate/up/down device pointers (packed or FP16/BF16
    row-major), their quant codes, the shared intermediate size and an
    optional fp32 [hidden] router (None: weight 1)."""
    _fields_ = [("gate_quant", C.c_uint32), ("up_quant", C.c_uint32), ("down_quant", C.c_uint32),
                ("gate", C.c_void_p), ("up", C.c_void_p), ("down", C.c_void_p), ("inter", C.c_uint32),
                ("router", C.c_void_p)]


def load() -> C.CDLL:
    """Load the in-tree library (raises if it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise Qw6CudaError(f"{LIB_PATH} is missing; build it with `make -C {CSRC}` (or __graft_entry__.build())")
    lib = C.CDLL(str(LIB_PATH))
    for name in ("qw6_vk_matmul_q4k_host", "qw6_vk_matmul_q5k_host", "qw6_vk_matmul_q6k_host",
                 "qw6_vk_matmul_iq2xxs_host", "qw6_vk_matmul_iq2s_host", "qw6_vk_matmul_iq3s_host"):
        getattr(lib, name).argtypes = [_u8p, _f32p, _f32p, _u32, _u32]
    lib.qw6_vk_matvec_f32_host.argtypes = [_f32p, _f32p, _f32p, _u32, _u32]
    lib.qw6_vk_silu_mul_host.argtypes = [_f32p, _f32p, _f32p, _u32]
    lib.qw6_vk_argmax_host.argtypes = [_f32p, _u32, C.POINTER(C.c_uint32), C.POINTER(C.c_float)]
    lib.qw6_vk_sampling_greedy_host.argtypes = [_f32p, _u32, C.POINTER(C.c_uint32)]
    lib.qw6_vk_moe_route_host.argtypes = [_f32p, _u32p, _f32p, _u32, _u32]
    lib.qw6_vk_moe_gather_host.argtypes = [_f32p, _f32p, _vp, C.c_float, _f32p, _u32, _u32]
    lib.qw6_vk_selftest.argtypes = []
    lib.qw6cu_last_error.restype = C.c_char_p
    lib.qw6cu_create.argtypes = [C.POINTER(_vp), C.c_int]
    lib.qw6cu_destroy.argtypes = [_vp]
    lib.qw6cu_destroy.restype = None
    lib.qw6cu_set_stream.argtypes = [_vp, _vp]
    lib.qw6cu_get_stream.argtypes = [_vp]
    lib.qw6cu_get_stream.restype = _vp
    lib.qw6cu_synchronize.argtypes = [_vp]
    lib.qw6cu_packed_bytes.argtypes = [_u32, _u32, _u32]
    lib.qw6cu_packed_bytes.restype = _sz
    lib.qw6cu_pack.argtypes = [_vp, _u32, _vp, _vp, _u32, _u32, _u32, _sz, _sz]
    lib.qw6cu_dequantize.argtypes = [_vp, _u32, _vp, _vp, _u32, _u32]
    lib.qw6cu_matvec.argtypes = [_vp, _u32, _vp, _vp, _vp, _u32, _u32, _u32]
    lib.qw6cu_matvec_f32.argtypes = [_vp, _vp, _vp, _vp, _u32, _u32]
    lib.qw6cu_moe_route.argtypes = [_vp, _vp, _u32, _u32, _u32, _vp, _vp]
    lib.qw6cu_silu_mul.argtypes = [_vp, _vp, _vp, _vp, _u32]
    lib.qw6cu_moe_gather.argtypes = [_vp, _vp, _vp, _vp, C.c_float, _vp, _u32, _u32]
    lib.qw6cu_argmax.argtypes = [_vp, _vp, _u32, _vp, _vp]
    pk = C.POINTER(ExpertPack)
    lib.qw6cu_moe_decode.argtypes = [_vp, pk, pk, pk, _vp, _vp, _vp, _u32, _u32, _u32, _u32, _u32]
    lib.qw6cu_moe_decode_hostio.argtypes = [_vp, pk, pk, pk, _vp, _vp, _vp, _u32, _u32, _u32, _u32, _u32]
    lib.qw6cu_moe_decode_noalloc.argtypes = [pk, pk, pk, _vp, _vp, _vp, _u32, _u32, _u32, _u32, _u32, _vp]
    lib.qw6cu_moe_prefill.argtypes = [_vp, pk, pk, pk, _vp, _vp, _vp, _u32, _u32, _u32, _u32, _u32]
    _pp = C.POINTER(_vp)
    lib.qw6cu_moe_prefill_hostio.argtypes = [_vp, pk, pk, pk, _pp, _pp, _pp, _u32, _u32, _u32, _u32, _u32, _u32]
    lib.qw6cu_gguf_open.argtypes = [C.c_char_p, C.POINTER(_vp)]
    lib.qw6cu_gguf_close.argtypes = [_vp]
    lib.qw6cu_gguf_close.restype = None
    lib.qw6cu_gguf_tensor_count.argtypes = [_vp]
    lib.qw6cu_gguf_tensor_count.restype = C.c_uint32
    lib.qw6cu_gguf_tensor_info.argtypes = [_vp, C.c_uint32, C.POINTER(GgufTensor)]
    lib.qw6cu_gguf_find.argtypes = [_vp, C.c_char_p]
    lib.qw6cu_gguf_upload_bytes.argtypes = [_vp, C.c_uint32]
    lib.qw6cu_gguf_upload_bytes.restype = _sz
    lib.qw6cu_gguf_upload.argtypes = [_vp, _vp, C.c_uint32, _vp, _sz, C.POINTER(ExpertPack)]
    lib.qw6cu_gguf_upload_moe.argtypes = [_vp, _vp, C.c_uint32, C.POINTER(MoeTable)]
    lib.qw6cu_moe_table_free.argtypes = [C.POINTER(MoeTable)]
    lib.qw6cu_moe_table_free.restype = None
    lib.qw6cu_sample.argtypes = [_vp, _vp, _u32, _u32, C.c_float, C.c_float, C.c_int, _vp, _vp]
    lib.qw6cu_decoder_create.argtypes = [_vp, C.POINTER(ModelTensor), _u32, _u32, _u32, C.POINTER(_vp)]
    lib.qw6cu_decoder_forward.argtypes = [_vp, _u32, _u32, _vp, _vp]
    lib.qw6cu_decoder_generate.argtypes = [_vp, _u32, _u32, _u32, _u32p]
    lib.qw6cu_decoder_logits.argtypes = [_vp, C.POINTER(C.c_uint32)]
    lib.qw6cu_decoder_logits.restype = _vp
    lib.qw6cu_decoder_reset.argtypes = [_vp]
    lib.qw6cu_decoder_device_bytes.argtypes = [_vp]
    lib.qw6cu_decoder_device_bytes.restype = _sz
    lib.qw6cu_decoder_destroy.argtypes = [_vp]
    lib.qw6cu_decoder_destroy.restype = None
    lib.qw6cu_moe_block.argtypes = [_vp, _vp, _vp, _vp, pk, pk, pk, C.POINTER(SharedExpert), _vp, _u32, _u32, _u32,
                                    _u32, _u32]
    lib.qw6cu_moe_expert_rows.argtypes = [_vp, pk, pk, pk, _vp, _vp, _vp, _u32, _u32, _u32, _u32]
    lib.qw6cu_ep_count.argtypes = [_vp, _vp, _u32, _u32, _vp, _vp]
    lib.qw6cu_ep_pack.argtypes = [_vp, _vp, _vp, _vp, _u32, _u32, _u32, _vp, _u32, _vp, _vp]
    lib.qw6cu_ep_expand.argtypes = [_vp, _vp, _u32, _u32, _vp]
    lib.qw6cu_ep_combine.argtypes = [_vp, _vp, _vp, _vp, _u32, _u32, _u32, _vp]
    lib.qw6cu_ep_handle_bytes.restype = _sz
    lib.qw6cu_ep_handle_bytes.argtypes = []
    lib.qw6cu_ep_create.argtypes = [_vp, _u32, _u32, _u32, _u32, _u32, _u32, _u32, C.POINTER(_vp)]
    lib.qw6cu_ep_handle.argtypes = [_vp, _vp]
    lib.qw6cu_ep_connect.argtypes = [_vp, _vp]
    lib.qw6cu_ep_layer.argtypes = [_vp, pk, pk, pk, _vp, _vp, _vp, _u32]
    lib.qw6cu_ep_layer_hostio.argtypes = [_vp, pk, pk, pk, C.POINTER(_vp), C.POINTER(_vp), C.POINTER(_vp), _u32,
                                          _u32]
    lib.qw6cu_ep_set_placement.argtypes = [_vp, _vp]
    lib.qw6cu_ep_last_rows.argtypes = [_vp, C.POINTER(_u32)]
    lib.qw6cu_ep_set_wait_limit.argtypes = [_vp, _u32]
    lib.qw6cu_ep_destroy.argtypes = [_vp]
    lib.qw6cu_ep_destroy.restype = None
    lib.qw6cu_moe_prefill_workspace_bytes.argtypes = [_u32, _u32, _u32, _u32, _u32]
    lib.qw6cu_moe_prefill_workspace_bytes.restype = _sz
    lib.qw6cu_gemm_bf16_nt.argtypes = [_vp, _vp, _vp, _vp, _u32, _u32, _u32]
    lib.qw6cu_check_device_errors.argtypes = [_vp]
    lib.qw6cu_lm_head_argmax.argtypes = [_vp, _u32, _vp, _vp, _u32, _u32, _u32, _u32, _vp, _vp]
    lib.qw6cu_argmax_keys_reduce.argtypes = [_vp, _vp, _u32, _u32, _vp, _vp]
    lib.qw6cu_profile_begin.argtypes = [_vp, _u32]
    lib.qw6cu_profile_end.argtypes = [_vp, C.POINTER(C.c_double), C.POINTER(C.c_uint32)]
    lib.qw6cu_kernel_name.argtypes = [C.c_int]
    lib.qw6cu_kernel_name.restype = C.c_char_p
    lib.qw6cu_moe_workspace_bytes.argtypes = [_u32, _u32, _u32, _u32, _u32]
    lib.qw6cu_moe_workspace_bytes.restype = _sz
    _lib = lib
    return lib


def last_error() -> str:
    msg = load().qw6cu_last_error()
    return msg.decode() if msg else ""


def _check(rc: int, what: str) -> None:
    if rc != 0:
        raise Qw6CudaError(f"{what} failed (rc={rc}): {last_error()}")


# ---------------------------------------------------------- qw6_vk.h -----

_MATMUL = {Q4_K: "q4k", Q4_K_S: "q4k", Q5_K: "q5k", Q6_K: "q6k", IQ2_XXS: "iq2xxs", IQ2_S: "iq2s", IQ3_S: "iq3s"}


def matmul_host(quant: int, w: np.ndarray, x: np.ndarray, rows: int, cols: int) -> np.ndarray:
    """qw6_vk_matmul_<fmt>_host: raw GGUF bytes + fp32 x -> fp32 y[rows]."""
    fn = getattr(load(), f"qw6_vk_matmul_{_MATMUL[quant]}_host")
    w = np.ascontiguousarray(w).view(np.uint8).reshape(-1)
    x = np.ascontiguousarray(x, np.float32).reshape(-1)
    y = np.empty(rows, np.float32)
    _check(fn(w, x, y, rows, cols), f"qw6_vk_matmul_{_MATMUL[quant]}_host")
    return y


def matvec_f32_host(w: np.ndarray, x: np.ndarray, rows: int, cols: int) -> np.ndarray:
    y = np.empty(rows, np.float32)
    _check(load().qw6_vk_matvec_f32_host(np.ascontiguousarray(w, np.float32).reshape(-1),
                                         np.ascontiguousarray(x, np.float32), y, rows, cols),
           "qw6_vk_matvec_f32_host")
    return y


def silu_mul_host(g: np.ndarray, u: np.ndarray) -> np.ndarray:
    g = np.ascontiguousarray(g, np.float32)
    out = np.empty_like(g)
    _check(load().qw6_vk_silu_mul_host(g, np.ascontiguousarray(u, np.float32), out, g.size), "silu_mul_host")
    return out


def argmax_host(x: np.ndarray):
    x = np.ascontiguousarray(x, np.float32)
    i, v = C.c_uint32(), C.c_float()
    _check(load().qw6_vk_argmax_host(x, x.size, C.byref(i), C.byref(v)), "argmax_host")
    return int(i.value), float(v.value)


def sampling_greedy_host(x: np.ndarray) -> int:
    x = np.ascontiguousarray(x, np.float32)
    t = C.c_uint32()
    _check(load().qw6_vk_sampling_greedy_host(x, x.size, C.byref(t)), "sampling_greedy_host")
    return int(t.value)


def moe_route_host(logits: np.ndarray, top_k: int):
    logits = np.ascontiguousarray(logits, np.float32)
    idx = np.empty(top_k, np.uint32)
    w = np.empty(top_k, np.float32)
    _check(load().qw6_vk_moe_route_host(logits, idx, w, logits.size, top_k), "moe_route_host")
    return idx, w


def moe_gather_host(expert_out, w, shared, shared_weight, dim, top_k):
    out = np.empty(dim, np.float32)
    sh = None if shared is None else np.ascontiguousarray(shared, np.float32)
    _check(load().qw6_vk_moe_gather_host(np.ascontiguousarray(expert_out, np.float32),
                                         np.ascontiguousarray(w, np.float32),
                                         None if sh is None else sh.ctypes.data, float(shared_weight), out,
                                         dim, top_k), "moe_gather_host")
    return out


def moe_decode_noalloc(gate: ExpertPack, up: ExpertPack, down: ExpertPack, logits, x, out, ntok, hidden, inter,
                       n_experts, top_k, stream=0) -> None:
    """qw6cu_moe_decode_noalloc: device pointers, caller's stream (0 = the
    legacy default stream), no device allocation; scratch is the library's
    fixed 1 MiB device array."""
    _check(load().qw6cu_moe_decode_noalloc(C.byref(gate), C.byref(up), C.byref(down), logits, x, out, ntok, hidden,
                                           inter, n_experts, top_k, stream or None), "qw6cu_moe_decode_noalloc")


def selftest() -> int:
    return int(load().qw6_vk_selftest())


# -------------------------------------------------------- qw6_cuda.h -----

class Context:
    """A qw6cu_ctx: one device, one stream (optionally an external one)."""

    def __init__(self, device: int = -1, stream: int | None = None) -> None:
        self.lib = load()
        h = _vp()
        _check(self.lib.qw6cu_create(C.byref(h), device), "qw6cu_create")
        self.h = h
        if stream is not None:
            self.set_stream(stream)

    def close(self) -> None:
        if self.h:
            self.lib.qw6cu_destroy(self.h)
            self.h = _vp()

    def __del__(self):  # pragma: no cover
        try:
            self.close()
        except Exception:
            pass

    def set_stream(self, stream: int | None) -> None:
        _check(self.lib.qw6cu_set_stream(self.h, stream or None), "qw6cu_set_stream")

    def synchronize(self) -> None:
        _check(self.lib.qw6cu_synchronize(self.h), "qw6cu_synchronize")

    @staticmethod
    def packed_bytes(quant: int, rows: int, cols: int) -> int:
        return int(load().qw6cu_packed_bytes(quant, rows, cols))

    def pack(self, quant, raw, packed, rows, cols, count=1, raw_stride=0, packed_stride=0):
        _check(self.lib.qw6cu_pack(self.h, quant, raw, packed, rows, cols, count, raw_stride, packed_stride),
               "qw6cu_pack")

    def dequantize(self, quant, raw, out, rows, cols):
        _check(self.lib.qw6cu_dequantize(self.h, quant, raw, out, rows, cols), "qw6cu_dequantize")

    def matvec(self, quant, packed, x, y, rows, cols, ntok=1):
        _check(self.lib.qw6cu_matvec(self.h, quant, packed, x, y, rows, cols, ntok), "qw6cu_matvec")

    def matvec_f32(self, w, x, y, rows, cols):
        _check(self.lib.qw6cu_matvec_f32(self.h, w, x, y, rows, cols), "qw6cu_matvec_f32")

    def moe_route(self, logits, ntok, n_experts, top_k, idx, w):
        _check(self.lib.qw6cu_moe_route(self.h, logits, ntok, n_experts, top_k, idx, w), "qw6cu_moe_route")

    def argmax(self, x, n, idx, val):
        _check(self.lib.qw6cu_argmax(self.h, x, n, idx, val), "qw6cu_argmax")

    def moe_decode(self, gate: ExpertPack, up: ExpertPack, down: ExpertPack, logits, x, out, ntok, hidden, inter,
                   n_experts, top_k):
        _check(self.lib.qw6cu_moe_decode(self.h, C.byref(gate), C.byref(up), C.byref(down), logits, x, out, ntok,
                                         hidden, inter, n_experts, top_k), "qw6cu_moe_decode")

    def moe_decode_hostio(self, gate: ExpertPack, up: ExpertPack, down: ExpertPack, logits, x, out, ntok, hidden,
                          inter, n_experts, top_k):
        """Host pointers (ints) for logits/x/out; synchronous."""
        _check(self.lib.qw6cu_moe_decode_hostio(self.h, C.byref(gate), C.byref(up), C.byref(down), logits, x, out,
                                                ntok, hidden, inter, n_experts, top_k), "qw6cu_moe_decode_hostio")

    def sample(self, logits, n, nrows, temp, top_p, top_k, u, token):
        """qw6cu_sample: device logits [nrows x n], device u [nrows] -> device
        token [nrows] (uint32)."""
        _check(self.lib.qw6cu_sample(self.h, logits, n, nrows, temp, top_p, top_k, u, token), "qw6cu_sample")

    def moe_block(self, x, norm_w, router, gate: ExpertPack, up: ExpertPack, down: ExpertPack,
                  shared: "SharedExpert | None", out, ntok, hidden, inter, n_experts, top_k):
        """qw6cu_moe_block: rmsnorm, fp32 router, routed experts, optional
        shared expert, residual (device pointers)."""
        _check(self.lib.qw6cu_moe_block(self.h, x, norm_w, router, C.byref(gate), C.byref(up), C.byref(down),
                                        C.byref(shared) if shared is not None else None, out, ntok, hidden, inter,
                                        n_experts, top_k), "qw6cu_moe_block")

    def moe_prefill(self, gate: ExpertPack, up: ExpertPack, down: ExpertPack, logits, x_bf16, out, ntok, hidden,
                    inter, n_experts, top_k):
        _check(self.lib.qw6cu_moe_prefill(self.h, C.byref(gate), C.byref(up), C.byref(down), logits, x_bf16, out,
                                          ntok, hidden, inter, n_experts, top_k), "qw6cu_moe_prefill")

    def moe_prefill_hostio(self, gate: ExpertPack, up: ExpertPack, down: ExpertPack, logits, x_bf16, out, ntok,
                           hidden, inter, n_experts, top_k):
        """qw6cu_moe_prefill_hostio: `logits`, `x_bf16`, `out` are equal-length
        sequences of HOST addresses, one entry per batch of ntok tokens."""
        n = len(logits)
        if len(x_bf16) != n or len(out) != n:
            raise ValueError("moe_prefill_hostio: logits, x_bf16 and out need one host address per batch")
        arr = lambda v: (_vp * max(n, 1))(*[int(p) for p in v])  # noqa: E731
        _check(self.lib.qw6cu_moe_prefill_hostio(self.h, C.byref(gate), C.byref(up), C.byref(down), arr(logits),
                                                 arr(x_bf16), arr(out), n, ntok, hidden, inter, n_experts, top_k),
               "qw6cu_moe_prefill_hostio")

    def moe_expert_rows(self, gate: ExpertPack, up: ExpertPack, down: ExpertPack, x_bf16, row_expert, out_bf16,
                        nrows, hidden, inter, n_experts):
        _check(self.lib.qw6cu_moe_expert_rows(self.h, C.byref(gate), C.byref(up), C.byref(down), x_bf16, row_expert,
                                              out_bf16, nrows, hidden, inter, n_experts), "qw6cu_moe_expert_rows")

    def ep_count(self, idx, nassign, n_experts, expert_count, pos):
        _check(self.lib.qw6cu_ep_count(self.h, idx, nassign, n_experts, expert_count, pos), "qw6cu_ep_count")

    def ep_pack(self, idx, pos, expert_count, nassign, top_k, n_experts, x_bf16, hidden, send_x, send_pos):
        _check(self.lib.qw6cu_ep_pack(self.h, idx, pos, expert_count, nassign, top_k, n_experts, x_bf16, hidden,
                                      send_x, send_pos), "qw6cu_ep_pack")

    def ep_expand(self, recv_count, world, experts_per_rank, row_expert):
        _check(self.lib.qw6cu_ep_expand(self.h, recv_count, world, experts_per_rank, row_expert), "qw6cu_ep_expand")

    def ep_combine(self, ret_bf16, w, send_pos, ntok, top_k, hidden, out):
        _check(self.lib.qw6cu_ep_combine(self.h, ret_bf16, w, send_pos, ntok, top_k, hidden, out), "qw6cu_ep_combine")

    def gemm_bf16_nt(self, A, B, D, M, N, K):
        _check(self.lib.qw6cu_gemm_bf16_nt(self.h, A, B, D, M, N, K), "qw6cu_gemm_bf16_nt")

    def check_device_errors(self):
        _check(self.lib.qw6cu_check_device_errors(self.h), "qw6cu_check_device_errors")

    def lm_head_argmax(self, quant, packed, x, ntok, rows, cols, row_offset, keys, logits=None):
        _check(self.lib.qw6cu_lm_head_argmax(self.h, quant, packed, x, ntok, rows, cols, row_offset, keys, logits),
               "qw6cu_lm_head_argmax")

    def argmax_keys_reduce(self, keys, nshards, ntok, idx, val=None):
        _check(self.lib.qw6cu_argmax_keys_reduce(self.h, keys, nshards, ntok, idx, val), "qw6cu_argmax_keys_reduce")

    def profile_begin(self, max_launches: int) -> None:
        _check(self.lib.qw6cu_profile_begin(self.h, max_launches), "qw6cu_profile_begin")

    def profile_end(self) -> dict:
        """{kernel name: (total ms, launches)} for the kernels that ran."""
        n = 21  # QW6CU_NKERNELS
        ms = (C.c_double * n)()
        cnt = (C.c_uint32 * n)()
        _check(self.lib.qw6cu_profile_end(self.h, ms, cnt), "qw6cu_profile_end")
        return {self.lib.qw6cu_kernel_name(i).decode(): (ms[i], cnt[i]) for i in range(n) if cnt[i]}

    @staticmethod
    def moe_workspace_bytes(ntok, hidden, inter, n_experts, top_k) -> int:
        return int(load().qw6cu_moe_workspace_bytes(ntok, hidden, inter, n_experts, top_k))


class PeerEP:
    """A qw6cu_ep: this rank's endpoint of the peer-memory expert-parallel
    MoE layer (experts sharded over `world` ranks: contiguously, or as
    `set_placement` says)."""

    def __init__(self, ctx: Context, rank: int, world: int, n_experts: int, top_k: int, hidden: int, inter: int,
                 max_tokens: int) -> None:
        self.ctx, self.lib = ctx, ctx.lib
        h = _vp()
        _check(self.lib.qw6cu_ep_create(ctx.h, rank, world, n_experts, top_k, hidden, inter, max_tokens, C.byref(h)),
               "qw6cu_ep_create")
        self.h = h

    @staticmethod
    def handle_bytes() -> int:
        return int(load().qw6cu_ep_handle_bytes())

    def handle(self) -> bytes:
        buf = C.create_string_buffer(self.handle_bytes())
        _check(self.lib.qw6cu_ep_handle(self.h, buf), "qw6cu_ep_handle")
        return buf.raw

    def connect(self, handles: list[bytes]) -> None:
        blob = b"".join(handles)
        _check(self.lib.qw6cu_ep_connect(self.h, C.c_char_p(blob)), "qw6cu_ep_connect")

    def layer(self, gate: ExpertPack, up: ExpertPack, down: ExpertPack, logits, x_bf16, out, ntok) -> None:
        _check(self.lib.qw6cu_ep_layer(self.h, C.byref(gate), C.byref(up), C.byref(down), logits, x_bf16, out, ntok),
               "qw6cu_ep_layer")

    def layer_hostio(self, gate: ExpertPack, up: ExpertPack, down: ExpertPack, logits, x_bf16, out, ntok) -> None:
        """qw6cu_ep_layer_hostio: `logits`, `x_bf16`, `out` are equal-length
        sequences of HOST addresses, one entry per layer step."""
        n = len(logits)
        if len(x_bf16) != n or len(out) != n:
            raise ValueError("layer_hostio: logits, x_bf16 and out need one host address per step")
        arr = lambda v: (_vp * max(n, 1))(*[int(p) for p in v])  # noqa: E731
        _check(self.lib.qw6cu_ep_layer_hostio(self.h, C.byref(gate), C.byref(up), C.byref(down), arr(logits),
                                              arr(x_bf16), arr(out), n, ntok), "qw6cu_ep_layer_hostio")

    def set_placement(self, experts) -> None:
        """experts: n_experts routed expert ids, rank r's local experts at
        [r*epr, (r+1)*epr) (the same on every rank)."""
        arr = (_u32 * len(experts))(*[int(e) for e in experts])
        _check(self.lib.qw6cu_ep_set_placement(self.h, arr), "qw6cu_ep_set_placement")

    def set_wait_limit(self, ms: int) -> None:
        """Give up every cross-GPU wait of later layers after `ms` ms."""
        _check(self.lib.qw6cu_ep_set_wait_limit(self.h, ms), "qw6cu_ep_set_wait_limit")

    def last_rows(self) -> int:
        r = _u32()
        _check(self.lib.qw6cu_ep_last_rows(self.h, C.byref(r)), "qw6cu_ep_last_rows")
        return int(r.value)

    def close(self) -> None:
        if self.h:
            self.lib.qw6cu_ep_destroy(self.h)
            self.h = _vp()

    def __del__(self):  # pragma: no cover
        try:
            self.close()
        except Exception:
            pass



class Gguf:
    """A GGUF file opened by the library (qw6cu_gguf_*): its tensor table,
    and uploads of tensors into device memory in the kernels' layout."""

    def __init__(self, path) -> None:
        self.lib = load()
        h = _vp()
        _check(self.lib.qw6cu_gguf_open(str(path).encode(), C.byref(h)), "qw6cu_gguf_open")
        self.h = h

    def close(self) -> None:
        if self.h:
            self.lib.qw6cu_gguf_close(self.h)
            self.h = _vp()

    def __del__(self):  # pragma: no cover
        try:
            self.close()
        except Exception:
            pass

    def __len__(self) -> int:
        return int(self.lib.qw6cu_gguf_tensor_count(self.h))

    def info(self, i: int) -> dict:
        t = GgufTensor()
        _check(self.lib.qw6cu_gguf_tensor_info(self.h, i, C.byref(t)), "qw6cu_gguf_tensor_info")
        return {"name": t.name.decode(), "dims": [int(t.dims[d]) for d in range(t.n_dims)],
                "ggml_type": int(t.ggml_type), "quant": int(t.quant), "file_offset": int(t.file_offset),
                "bytes": int(t.bytes)}

    def find(self, name: str) -> int:
        return int(self.lib.qw6cu_gguf_find(self.h, name.encode()))

    def upload_bytes(self, i: int) -> int:
        return int(self.lib.qw6cu_gguf_upload_bytes(self.h, i))

    def upload(self, ctx: "Context", i: int, dst: int, dst_bytes: int) -> ExpertPack:
        p = ExpertPack()
        _check(self.lib.qw6cu_gguf_upload(ctx.h, self.h, i, dst, dst_bytes, C.byref(p)), "qw6cu_gguf_upload")
        return p

    def upload_moe(self, ctx: "Context", n_layers: int) -> MoeTable:
        t = MoeTable()
        _check(self.lib.qw6cu_gguf_upload_moe(ctx.h, self.h, n_layers, C.byref(t)), "qw6cu_gguf_upload_moe")
        return t

    def layer_packs(self, table: MoeTable, layer: int) -> tuple:
        arr = C.cast(table.packs, C.POINTER(ExpertPack))
        return tuple(ExpertPack(arr[3 * layer + k].quant, arr[3 * layer + k].base, arr[3 * layer + k].stride)
                     for k in range(3))

    def free_table(self, table: MoeTable) -> None:
        self.lib.qw6cu_moe_table_free(C.byref(table))


class Decoder:
    """qw6cu_decoder: qw6's per-token forward pass on the device, replayed
    as one CUDA graph per step.  `model` is a qw6_b200.synth.FwdModel-like
    object: n_layers and .tensors of (field, layer, quant, rows, cols, host
    array, stride); its arrays must stay alive until create() returns (the
    decoder keeps device copies)."""

    def __init__(self, ctx: "Context", model, max_ctx: int) -> None:
        self.lib = ctx.lib
        self.ctx = ctx
        ts = (ModelTensor * len(model.tensors))()
        for i, (f, l, q, r, c, arr, stride) in enumerate(model.tensors):
            ts[i] = ModelTensor(f, l, q, r, c, arr.ctypes.data, stride)
        h = _vp()
        _check(self.lib.qw6cu_decoder_create(ctx.h, ts, len(model.tensors), model.n_layers, max_ctx, C.byref(h)),
               "qw6cu_decoder_create")
        self.h = h
        n = C.c_uint32()
        self.lib.qw6cu_decoder_logits(self.h, C.byref(n))
        self.vocab = int(n.value)

    def close(self) -> None:
        if self.h:
            self.lib.qw6cu_decoder_destroy(self.h)
            self.h = _vp()

    def __del__(self):  # pragma: no cover
        try:
            self.close()
        except Exception:
            pass

    def forward(self, token: int, pos: int, logits: bool = True):
        """One step: (logits [vocab] or None, greedy token id)."""
        out = np.empty(self.vocab, np.float32) if logits else None
        g = C.c_uint32()
        _check(self.lib.qw6cu_decoder_forward(self.h, token, pos, out.ctypes.data if logits else None, C.byref(g)),
               "qw6cu_decoder_forward")
        return out, int(g.value)

    def generate(self, token: int, pos: int, n: int) -> np.ndarray:
        out = np.empty(n, np.uint32)
        _check(self.lib.qw6cu_decoder_generate(self.h, token, pos, n, out), "qw6cu_decoder_generate")
        return out

    def logits_ptr(self) -> int:
        return int(self.lib.qw6cu_decoder_logits(self.h, None) or 0)

    def reset(self) -> None:
        _check(self.lib.qw6cu_decoder_reset(self.h), "qw6cu_decoder_reset")

    def device_bytes(self) -> int:
        return int(self.lib.qw6cu_decoder_device_bytes(self.h))
