"""ctypes front-end of the CPU checkers.  TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import
this module.  Two checkers are exposed with the same call shapes:

* ``Oracle()``     -- liboracle.so, the C restatement of qw6's CPU path.
* ``Reference()``  -- oracle/_ref/libqw6ref.so, qw6's own qw6.c compiled
                      from its sources (present when it was built here).
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ORACLE_SO = HERE / "liboracle.so"
REF_SO = HERE / "_ref" / "libqw6ref.so"

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C")
_f64p = np.ctypeslib.ndpointer(np.float64, flags="C")
_i32p = np.ctypeslib.ndpointer(np.int32, flags="C")
_u32p = np.ctypeslib.ndpointer(np.uint32, flags="C")


def build() -> None:
    """Build liboracle.so (and _ref when the reference tree is present)."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)


def _load(path: Path) -> C.CDLL:
    if not path.exists():
        build()
    return C.CDLL(str(path))


def _u8(a: np.ndarray) -> np.ndarray:
    a = np.ascontiguousarray(a)
    return a.view(np.uint8) if a.dtype != np.uint8 else a


class _ExpertPack(C.Structure):
    _fields_ = [("quant", C.c_uint32), ("base", C.c_void_p), ("stride", C.c_size_t)]


class _Matrix(C.Structure):
    _fields_ = [("quant", C.c_uint32), ("w", C.c_void_p)]


class Oracle:
    """C restatement (qw6_oracle.c)."""

    kind = "port"

    def __init__(self) -> None:
        lib = _load(ORACLE_SO)
        lib.qo_dequantize_row.argtypes = [C.c_uint32, C.c_void_p, C.c_uint32, C.c_uint32, _f32p]
        lib.qo_matvec.argtypes = [C.c_uint32, C.c_void_p, _f32p, _f32p, C.c_uint32, C.c_uint32]
        lib.qo_matvec_f64.argtypes = [C.c_uint32, C.c_void_p, _f32p, _f64p, C.c_uint32, C.c_uint32]
        lib.qo_matvec_batch.argtypes = [C.c_uint32, C.c_void_p, _f32p, _f32p, C.c_uint32,
                                        C.c_uint32, C.c_uint32]
        lib.qo_moe_route.argtypes = [_f32p, C.c_uint32, C.c_uint32, _i32p, _f32p]
        lib.qo_argmax.argtypes = [_f32p, C.c_uint32]
        lib.qo_argmax.restype = C.c_int32
        lib.qo_fp16_to_f32.argtypes = [C.c_uint16]
        lib.qo_fp16_to_f32.restype = C.c_float
        lib.qo_moe_gather.argtypes = [_f32p, _f32p, C.c_void_p, C.c_float, _f32p, C.c_uint32, C.c_uint32]
        lib.qo_silu_mul.argtypes = [_f32p, _f32p, _f32p, C.c_uint32]
        pk = C.POINTER(_ExpertPack)
        lib.qo_moe_layer.argtypes = [pk, pk, pk, _f32p, _f32p, _f32p, C.c_uint32, C.c_uint32,
                                     C.c_uint32, C.c_uint32, C.c_uint32, C.c_void_p, C.c_void_p]
        lib.qo_moe_layer_f64.argtypes = [pk, pk, pk, _f32p, _f32p, _f64p, C.c_uint32, C.c_uint32,
                                         C.c_uint32, C.c_uint32, C.c_uint32]
        lib.qo_rmsnorm.argtypes = [_f32p, _f32p, _f32p, C.c_uint32]
        lib.qo_rmsnorm.restype = None
        lib.qo_sample.argtypes = [_f32p, C.c_uint32, C.c_float, C.c_float, C.c_int, C.c_float]
        lib.qo_fwd_state_floats.argtypes = [C.c_uint32, C.c_uint32]
        lib.qo_fwd_state_floats.restype = C.c_size_t
        lib.qo_forward.argtypes = [C.c_void_p, _f32p, C.c_uint32, C.c_uint32, C.c_uint32, _f32p]
        lib.qo_sample.restype = C.c_int32
        mp = C.POINTER(_Matrix)
        lib.qo_moe_block.argtypes = [_f32p, _f32p, mp, pk, pk, pk, mp, mp, mp, mp, _f32p, C.c_uint32, C.c_uint32,
                                     C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32]
        lib.qo_moe_block_f64.argtypes = [_f32p, _f32p, mp, pk, pk, pk, mp, mp, mp, mp, _f64p, C.c_uint32,
                                         C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32]
        self.lib = lib

    def fp16_to_f32(self, h: int) -> float:
        return self.lib.qo_fp16_to_f32(h)

    def dequantize(self, quant: int, w: np.ndarray, rows: int, cols: int) -> np.ndarray:
        w = _u8(w)
        out = np.empty((rows, cols), np.float32)
        for r in range(rows):
            if self.lib.qo_dequantize_row(quant, w.ctypes.data, cols, r, out[r]):
                raise ValueError("dequantize_row failed")
        return out

    def matvec(self, quant: int, w: np.ndarray, x: np.ndarray, rows: int, cols: int) -> np.ndarray:
        w = _u8(w)
        x = np.ascontiguousarray(x, np.float32).reshape(-1)
        ntok = x.size // cols
        y = np.empty(ntok * rows, np.float32)
        if self.lib.qo_matvec_batch(quant, w.ctypes.data, x, y, rows, cols, ntok):
            raise ValueError("matvec failed")
        return y.reshape(ntok, rows) if ntok > 1 else y

    def matvec_f64(self, quant: int, w: np.ndarray, x: np.ndarray, rows: int, cols: int) -> np.ndarray:
        w = _u8(w)
        x = np.ascontiguousarray(x, np.float32).reshape(-1)
        y = np.empty(rows, np.float64)
        if self.lib.qo_matvec_f64(quant, w.ctypes.data, x, y, rows, cols):
            raise ValueError("matvec_f64 failed")
        return y

    def moe_layer_grouped_f64(self, gq, gate, up, dq, down, logits, x, top_k=8):
        """Float64 recomputation of the routed-MoE layer (qw6.c:2246-2264) for a
        whole token batch, grouped by expert: the routing (indices and fp32
        softmax weights) is the oracle's bit-exact qw6_cpu_moe_route, every
        expert's weights are the oracle's bit-exact dequantization widened to
        float64, and each expert's rows are one float64 matmul per projection,
        so a batch of thousands of tokens takes seconds.  Returns (out [ntok,
        hidden] float64, idx, w)."""
        logits = np.ascontiguousarray(logits, np.float32)
        x = np.ascontiguousarray(x, np.float32).astype(np.float64)
        ntok, hidden = x.shape
        inter = gate.shape[1]
        idx = np.empty((ntok, top_k), np.int32)
        w = np.empty((ntok, top_k), np.float32)
        for t in range(ntok):
            idx[t], w[t] = self.moe_route(logits[t], top_k)
        out = np.zeros((ntok, hidden), np.float64)
        flat = idx.reshape(-1)
        order = np.argsort(flat, kind="stable")
        bounds = np.searchsorted(flat[order], np.arange(gate.shape[0] + 1))
        for e in range(gate.shape[0]):
            sel = order[bounds[e]:bounds[e + 1]]
            if sel.size == 0:
                continue
            tok = sel // top_k
            wg = self.dequantize(gq, gate[e], inter, hidden).astype(np.float64)
            wu = self.dequantize(gq, up[e], inter, hidden).astype(np.float64)
            wd = self.dequantize(dq, down[e], hidden, inter).astype(np.float64)
            xe = x[tok]
            g, u = xe @ wg.T, xe @ wu.T
            with np.errstate(over="ignore"):  # exp(-g) = inf for very negative g: silu -> 0, as intended
                mid = g / (1.0 + np.exp(-g)) * u
            np.add.at(out, tok, (mid @ wd.T) * w.reshape(-1)[sel].astype(np.float64)[:, None])
        return out, idx, w

    def moe_route(self, logits: np.ndarray, top_k: int):
        logits = np.ascontiguousarray(logits, np.float32)
        idx = np.empty(top_k, np.int32)
        w = np.empty(top_k, np.float32)
        if self.lib.qo_moe_route(logits, logits.size, top_k, idx, w):
            raise ValueError("moe_route failed")
        return idx, w

    def argmax(self, x: np.ndarray) -> int:
        x = np.ascontiguousarray(x, np.float32)
        return int(self.lib.qo_argmax(x, x.size))

    def moe_gather(self, expert_out, w, shared, shared_weight, dim, top_k):
        out = np.empty(dim, np.float32)
        sh = None if shared is None else np.ascontiguousarray(shared, np.float32)
        self.lib.qo_moe_gather(np.ascontiguousarray(expert_out, np.float32),
                               np.ascontiguousarray(w, np.float32),
                               None if sh is None else sh.ctypes.data, float(shared_weight),
                               out, dim, top_k)
        return out

    def silu_mul(self, g, u):
        g = np.ascontiguousarray(g, np.float32)
        u = np.ascontiguousarray(u, np.float32)
        out = np.empty_like(g)
        self.lib.qo_silu_mul(g, u, out, g.size)
        return out

    @staticmethod
    def _pack(quant, arr):
        arr = _u8(arr)
        return _ExpertPack(quant, arr.ctypes.data, arr[0].nbytes), arr

    def forward(self, model, tokens, max_ctx=None):
        """qo_forward (qw6_forward_token, qw6.c:2426-2500) over tokens at
        positions 0.. from a cleared state: [n, model.vocab] logits."""
        return _forward_oracle(self.lib, model, tokens, max_ctx or len(tokens))

    def sample(self, logits, temp, top_p, top_k, u):
        """qw6_sample (qw6.c:2921-2982) with its uniform draw u given."""
        logits = np.ascontiguousarray(logits, np.float32)
        return int(self.lib.qo_sample(logits, logits.size, temp, top_p, top_k, u))

    def rmsnorm(self, x, w):
        """qw6_cpu_rmsnorm (qw6.c:2502-2512)."""
        x = np.ascontiguousarray(x, np.float32)
        w = np.ascontiguousarray(w, np.float32)
        out = np.empty_like(x)
        self.lib.qo_rmsnorm(x, w, out, x.size)
        return out

    def moe_block(self, x, norm_w, router, experts, shared=None, top_k=8, f64=False):
        """The MoE FFN block around qw6_apply_layer_moe (qw6.c:2474-2484,
        2226-2290) for every token row of x: rmsnorm, router matvec, routed
        experts, the optional shared expert with its sigmoid gate, residual
        add.  router: (quant, matrix [n_experts rows]); experts: (gq, gate,
        up, dq, down) as for moe_layer; shared: None or ((quant, gate),
        (quant, up), (quant, down), (quant, router) or None).  f64: the
        double-precision error reference (same routing)."""
        gq, gate, up, dq, down = experts
        x = np.ascontiguousarray(x, np.float32)
        ntok, hidden = x.shape
        norm_w = np.ascontiguousarray(norm_w, np.float32)
        keep = []

        def mat(qm):
            if qm is None:
                return None
            arr = _u8(qm[1])
            keep.append(arr)
            return C.byref(_Matrix(qm[0], arr.ctypes.data))

        pg, _a = self._pack(gq, gate)
        pu, _b = self._pack(gq, up)
        pd, _c = self._pack(dq, down)
        sg, su, sd, sr = shared if shared is not None else (None, None, None, None)
        shared_inter = np.asarray(sg[1]).shape[0] if sg is not None else 0
        out = np.empty(x.shape, np.float64 if f64 else np.float32)
        fn = self.lib.qo_moe_block_f64 if f64 else self.lib.qo_moe_block
        rc = fn(x, norm_w, mat(router), C.byref(pg), C.byref(pu), C.byref(pd), mat(sg), mat(su), mat(sd), mat(sr),
                out, ntok, hidden, gate.shape[1], shared_inter, gate.shape[0], top_k)
        if rc:
            raise ValueError("moe_block failed")
        return out

    def moe_layer(self, gq, gate, up, dq, down, logits, x, top_k=8, f64=False):
        """Routed MoE FFN (qw6.c:2246-2264) for every token row of x."""
        logits = np.ascontiguousarray(logits, np.float32)
        x = np.ascontiguousarray(x, np.float32)
        ntok, hidden = x.shape
        n_experts = logits.shape[1]
        inter = gate.shape[1]
        pg, _a = self._pack(gq, gate)
        pu, _b = self._pack(gq, up)
        pd, _c = self._pack(dq, down)
        if f64:
            out = np.empty((ntok, hidden), np.float64)
            rc = self.lib.qo_moe_layer_f64(C.byref(pg), C.byref(pu), C.byref(pd), logits, x, out,
                                           ntok, hidden, inter, n_experts, top_k)
            if rc:
                raise ValueError("moe_layer_f64 failed")
            return out
        out = np.empty((ntok, hidden), np.float32)
        idx = np.empty((ntok, top_k), np.int32)
        w = np.empty((ntok, top_k), np.float32)
        rc = self.lib.qo_moe_layer(C.byref(pg), C.byref(pu), C.byref(pd), logits, x, out, ntok,
                                   hidden, inter, n_experts, top_k, idx.ctypes.data, w.ctypes.data)
        if rc:
            raise ValueError("moe_layer failed")
        return out, idx, w


class _Tensor(C.Structure):
    _fields_ = [("quant", C.c_uint32), ("rows", C.c_uint32), ("cols", C.c_uint32), ("data", C.c_void_p),
                ("stride", C.c_size_t)]


class _Model(C.Structure):
    _fields_ = [("n_layers", C.c_uint32), ("tok_embd", _Tensor), ("output", _Tensor), ("output_norm", _Tensor),
                ("layers", C.c_void_p)]


N_FIELDS = 24  # per-layer roles (QO_F_* / QW6CU_F_*)


def _forward_oracle(lib, model, tokens, max_ctx):
    """qo_forward over tokens at positions 0.. (fresh state): [n, vocab] logits."""
    layers = (_Tensor * (model.n_layers * N_FIELDS))()
    glob = {}
    for f, l, q, r, c, arr, stride in model.tensors:
        t = _Tensor(q, r, c, arr.ctypes.data, stride)
        if l < 0:
            glob[f] = t
        else:
            layers[l * N_FIELDS + f] = t
    m = _Model(model.n_layers, glob[100], glob[101], glob[102], C.cast(layers, C.c_void_p))
    state = np.zeros(lib.qo_fwd_state_floats(model.n_layers, max_ctx), np.float32)
    out = np.zeros((len(tokens), model.vocab), np.float32)
    for pos, tok in enumerate(tokens):
        if lib.qo_forward(C.byref(m), state, max_ctx, int(tok), pos, out[pos]):
            raise ValueError(f"qo_forward failed at position {pos}")
    return out


class _RefModel:
    """A qw6_model_t built by the shim of a reference library from a model's
    tensors (which must outlive it)."""

    def __init__(self, lib, model):
        self.lib, self.model = lib, model
        self.h = lib.ref_model_new()
        for f, l, q, r, c, arr, stride in model.tensors:
            if lib.ref_model_set(self.h, l, f, q, r, c, arr.ctypes.data, stride):
                raise ValueError(f"ref_model_set rejected field {f} layer {l}")

    def close(self):
        if self.h:
            self.lib.ref_model_free(self.h)
            self.h = None


def _bind_model_shim(lib):
    lib.ref_model_new.restype = C.c_void_p
    lib.ref_model_set.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_uint32, C.c_uint32, C.c_void_p,
                                  C.c_size_t]
    lib.ref_model_free.argtypes = [C.c_void_p]
    lib.ref_forward.argtypes = [C.c_void_p, _u32p, C.c_uint32, _f32p, C.c_uint32, C.c_int]


def _ref_forward(lib, model, tokens, use_pipe=False):
    """qw6_prefill one token at a time through qw6's session (qw6.c:2867-2882)."""
    tok = np.ascontiguousarray(tokens, np.uint32)
    out = np.zeros((tok.size, model.vocab), np.float32)
    rm = _RefModel(lib, model)
    try:
        rc = lib.ref_forward(rm.h, tok, tok.size, out, model.vocab, int(use_pipe))
    finally:
        rm.close()
    if rc:
        raise ValueError("qw6's forward pass returned an error")
    return out


class Reference:
    """qw6's own CPU functions, compiled from its sources (oracle/_ref)."""

    kind = "reference"

    @staticmethod
    def available() -> bool:
        return REF_SO.exists()

    def __init__(self) -> None:
        if not REF_SO.exists():
            build()
        lib = C.CDLL(str(REF_SO))
        lib.ref_dequantize_row.argtypes = [C.c_int, C.c_void_p, C.c_uint32, C.c_uint32, C.c_uint32, _f32p]
        lib.ref_matvec.argtypes = [C.c_int, C.c_void_p, _f32p, _f32p, C.c_uint32, C.c_uint32]
        lib.ref_moe_route.argtypes = [_f32p, C.c_int, C.c_int, _i32p, _f32p]
        lib.ref_argmax.argtypes = [_f32p, C.c_int]
        lib.ref_silu.argtypes = [C.c_float]
        lib.ref_silu.restype = C.c_float
        lib.ref_sigmoid.argtypes = [C.c_float]
        lib.ref_sigmoid.restype = C.c_float
        lib.ref_rmsnorm.argtypes = [_f32p, _f32p, _f32p, C.c_int]
        lib.ref_sample.argtypes = [_f32p, C.c_float, C.c_float, C.c_int, C.c_uint]
        lib.ref_rand_unit.argtypes = [C.c_uint]
        lib.ref_rand_unit.restype = C.c_float
        lib.ref_moe_tokens.argtypes = [C.c_int, C.c_void_p, C.c_void_p, C.c_size_t, C.c_int, C.c_void_p, C.c_size_t,
                                       C.c_void_p, C.c_void_p, C.c_void_p, C.c_uint32, C.c_uint32, C.c_uint32,
                                       C.c_uint32, C.c_int, C.c_int]
        _bind_model_shim(lib)
        self.lib = lib
        self.vocab = int(lib.ref_vocab_size())

    def forward(self, model, tokens):
        """qw6's CPU forward pass (qw6_forward_token, qw6.c:2426-2500) over
        tokens at positions 0..: [n, model.vocab] logits.  qw6 runs its 40
        layers, so the model must have 40."""
        assert model.n_layers == 40
        return _ref_forward(self.lib, model, tokens)

    def dequantize(self, quant, w, rows, cols):
        w = _u8(w)
        out = np.empty((rows, cols), np.float32)
        for r in range(rows):
            if self.lib.ref_dequantize_row(quant, w.ctypes.data, rows, cols, r, out[r]):
                raise ValueError("ref dequantize failed")
        return out

    def matvec(self, quant, w, x, rows, cols):
        w = _u8(w)
        x = np.ascontiguousarray(x, np.float32).reshape(-1)
        ntok = x.size // cols
        y = np.empty((ntok, rows), np.float32)
        for t in range(ntok):
            if self.lib.ref_matvec(quant, w.ctypes.data, np.ascontiguousarray(x[t * cols:(t + 1) * cols]),
                                   y[t], rows, cols):
                raise ValueError("ref matvec failed")
        return y if ntok > 1 else y[0]

    def matvec_rows(self, quant, w_rows, x, rows, cols):
        """matvec over a contiguous slice of rows (bounded CPU samples)."""
        return self.matvec(quant, w_rows, x, rows, cols)

    def moe_tokens(self, gq, gate, up, dq, down, logits, x, t0, t1, top_k=8):
        """Tokens [t0, t1) of the routed-MoE layer through qw6's own expert loop
        (qw6.c:2246-2264) run entirely in C; gate/up/down are expert packs
        [n_experts, rows, row_bytes], logits [ntok, n_experts], x [ntok, hidden].
        Returns out rows [t1 - t0, hidden]."""
        gate, up, down = (np.ascontiguousarray(a).view(np.uint8) for a in (gate, up, down))
        logits = np.ascontiguousarray(logits[t0:t1], np.float32)
        x = np.ascontiguousarray(x[t0:t1], np.float32)
        ne, hidden, inter = logits.shape[1], x.shape[1], up.shape[1]
        out = np.zeros_like(x)
        rc = self.lib.ref_moe_tokens(gq, gate.ctypes.data, up.ctypes.data, gate[0].nbytes, dq, down.ctypes.data,
                                     down[0].nbytes, logits.ctypes.data, x.ctypes.data, out.ctypes.data, 0,
                                     t1 - t0, hidden, inter, ne, top_k)
        if rc:
            raise ValueError("ref moe_tokens failed")
        return out

    def moe_route(self, logits, top_k):
        logits = np.ascontiguousarray(logits, np.float32)
        idx = np.empty(top_k, np.int32)
        w = np.empty(top_k, np.float32)
        if self.lib.ref_moe_route(logits, logits.size, top_k, idx, w):
            raise ValueError("ref moe_route failed")
        return idx, w

    def argmax(self, x):
        x = np.ascontiguousarray(x, np.float32)
        return int(self.lib.ref_argmax(x, x.size))

    def silu(self, v: float) -> float:
        return self.lib.ref_silu(v)

    def sigmoid(self, v: float) -> float:
        return self.lib.ref_sigmoid(v)

    def sample(self, logits, temp, top_p, top_k, seed):
        """qw6_sample over qw6's full vocabulary row, libc rand() seeded with seed."""
        logits = np.ascontiguousarray(logits, np.float32)
        if logits.size != self.vocab:
            raise ValueError(f"qw6_sample reads {self.vocab} logits")
        return int(self.lib.ref_sample(logits, temp, top_p, top_k, seed))

    def rand_unit(self, seed) -> float:
        """The uniform draw qw6_sample makes after srand(seed)."""
        return float(self.lib.ref_rand_unit(seed))

    def rmsnorm(self, x, w):
        x = np.ascontiguousarray(x, np.float32)
        w = np.ascontiguousarray(w, np.float32)
        out = np.empty_like(x)
        if self.lib.ref_rmsnorm(x, w, out, x.size):
            raise ValueError("ref rmsnorm failed")
        return out

    def moe_block(self, x, norm_w, router, experts, shared=None, top_k=8):
        """qw6.c:2474-2484 around qw6_apply_layer_moe (qw6.c:2226-2290),
        composed from qw6's own functions in its order (same arguments as
        Oracle.moe_block)."""
        gq, gate, up, dq, down = experts
        x = np.ascontiguousarray(x, np.float32)
        ntok, hidden = x.shape
        ne = gate.shape[0]
        out = np.empty_like(x)
        for t in range(ntok):
            normed = self.rmsnorm(x[t], norm_w)
            logits = self.matvec(router[0], router[1], normed, ne, hidden)
            ffn = self.moe_layer(gq, gate, up, dq, down, logits[None, :], normed[None, :], top_k)[0][0]
            if shared is not None:
                (sgq, sgw), (suq, suw), (sdq, sdw), sr = shared
                s = np.float32(1.0)
                if sr is not None:
                    s = np.float32(self.sigmoid(float(np.atleast_1d(self.matvec(sr[0], sr[1], normed, 1, hidden))[0])))
                si = np.asarray(sgw).shape[0]
                g = self.matvec(sgq, sgw, normed, si, hidden)
                u = self.matvec(suq, suw, normed, si, hidden)
                mid = np.array([self.silu(float(v)) for v in g], np.float32) * u
                d = self.matvec(sdq, sdw, mid.astype(np.float32), hidden, si)
                ffn = (ffn + s * d).astype(np.float32)
            out[t] = (x[t] + ffn).astype(np.float32)
        return out

    def moe_layer(self, gq, gate, up, dq, down, logits, x, top_k=8):
        """qw6.c:2246-2264 composed from qw6's own public functions."""
        logits = np.ascontiguousarray(logits, np.float32)
        x = np.ascontiguousarray(x, np.float32)
        ntok, hidden = x.shape
        inter = gate.shape[1]
        out = np.zeros((ntok, hidden), np.float32)
        idxs = np.empty((ntok, top_k), np.int32)
        ws = np.empty((ntok, top_k), np.float32)
        for t in range(ntok):
            idx, w = self.moe_route(logits[t], top_k)
            idxs[t], ws[t] = idx, w
            acc = np.zeros(hidden, np.float32)
            for k in range(top_k):
                e = int(idx[k])
                g = self.matvec(gq, gate[e], x[t], inter, hidden)
                u = self.matvec(gq, up[e], x[t], inter, hidden)
                mid = np.array([self.silu(float(v)) for v in g], np.float32) * u
                d = self.matvec(dq, down[e], mid.astype(np.float32), hidden, inter)
                acc = (acc + np.float32(w[k]) * d).astype(np.float32)
            out[t] = acc
        return out, idxs, ws


def cpu_count() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:  # pragma: no cover
        return os.cpu_count() or 1


VK_SO = HERE / "_ref" / "libqw6vk.so"


class VkReference:
    """qw6.c built with QW6_VULKAN against include/qw6_vk.h and linked with
    libqw6cuda.so (oracle/_ref/libqw6vk.so): qw6's own session and forward
    pass, on its CPU path or through the qw6_vk_pipe_* entry points that this
    library provides (qw6_forward_token's pipeline branch, qw6.c:2429-2445)."""

    @staticmethod
    def available() -> bool:
        return VK_SO.exists()

    def __init__(self) -> None:
        lib = C.CDLL(str(VK_SO))
        _bind_model_shim(lib)
        lib.ref_pipe_greedy.argtypes = [C.c_void_p, _u32p, C.c_uint32, _u32p, C.c_void_p, C.c_uint32]
        self.lib = lib

    def forward(self, model, tokens, use_pipe: bool):
        assert model.n_layers == 40
        return _ref_forward(self.lib, model, tokens, use_pipe)

    def pipe_greedy(self, model, tokens, with_logits=True):
        """qw6_vk_pipe_forward_greedy per token: (picked ids, logits or None)."""
        tok = np.ascontiguousarray(tokens, np.uint32)
        picked = np.zeros(tok.size, np.uint32)
        out = np.zeros((tok.size, model.vocab), np.float32) if with_logits else None
        rm = _RefModel(self.lib, model)
        try:
            rc = self.lib.ref_pipe_greedy(rm.h, tok, tok.size, picked, out.ctypes.data if with_logits else None,
                                          model.vocab)
        finally:
            rm.close()
        if rc:
            raise ValueError("qw6_vk_pipe_forward_greedy failed")
        return picked, out
