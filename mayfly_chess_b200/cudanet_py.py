"""libcudanet_b200.so from Python through ctypes: the reference backend's Python interface, unchanged.

    net = CudaNet("net.cnw")
    pol, val, qv = net.evaluate(ids, cast, hm, ep, I, M)

This mirrors mayfly/chess/cudanet/cudanet_py.py:87-178 (class CudaNet): the same constructor
(weights_path, device=0, dll=None), the same evaluate(ids, cast, hm, ep, I, M) -> (pol, val, qv) with the same
shape and dtype checks (bool M is taken too), fingerprint(), profile(B, reps), close() and the context
manager, the same exceptions (ValueError for bad shapes or batch sizes, RuntimeError with the library's reason
for a failed call). The inputs are what MCTS._prepare builds: ids (B, 64) int64, cast (B, 4) float32, hm (B,)
int64, ep (B,) int64, I (B, wide) int64 and M (B, wide) uint8. The outputs are float32 pol (B, wide) (raw policy
logits at each row's legal moves, 0 on padding), val (B,) and qv (B, wide).

Additions: evaluate_logits (also the full (B, 8324) logits), begin/end (two batches in flight),
evaluate_device (torch CUDA tensors in and out, queued on a stream), precision, check, calibrate (the input
ranges an e4m3 weight file's static scales come from), and k_* single-kernel entry points for unit tests.

The library is MAYFLY_CUDANET_DLL, else libcudanet_b200.so beside this file. There is no fallback: if the
library is missing the constructor raises.
"""
import ctypes
import os
import threading

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
MAX_BATCH = 1024        # the library's default (env MAYFLY_CUDANET_MAX_BATCH when a net is made)
MAX_WIDE = 256
N_MOVES = 4162
ERR_LEN = 2048

_libs = {}
_load_lock = threading.Lock()


def dll_path(dll=None):
    """Which library file a handle binds: the explicit argument, then $MAYFLY_CUDANET_DLL, then the build in this
    package's folder."""
    for choice in (dll, os.environ.get("MAYFLY_CUDANET_DLL")):
        if choice:
            return choice
    return os.path.join(HERE, "libcudanet_b200.so")


def load(dll=None):
    """The library, loaded once per path, with every entry point's signature declared."""
    path = os.path.abspath(dll_path(dll))
    with _load_lock:
        if path in _libs:
            return _libs[path]
        if not os.path.exists(path):
            raise FileNotFoundError(f"no libcudanet_b200.so at {path} (build it: python -m mayfly_chess_b200.build)")
        lib = ctypes.CDLL(path)
        vp, i32, cp = ctypes.c_void_p, ctypes.c_int, ctypes.c_char_p
        lib.cudanet_create.argtypes = [cp, i32, cp, i32]
        lib.cudanet_create.restype = vp
        lib.cudanet_evaluate.argtypes = [vp, i32, i32] + [vp] * 9 + [cp, i32]
        lib.cudanet_evaluate.restype = i32
        lib.cudanet_evaluate_logits.argtypes = [vp, i32, i32] + [vp] * 10 + [cp, i32]
        lib.cudanet_evaluate_logits.restype = i32
        lib.cudanet_begin.argtypes = [vp, i32, i32] + [vp] * 6 + [cp, i32]
        lib.cudanet_begin.restype = i32
        lib.cudanet_end.argtypes = [vp, vp, vp, vp, cp, i32]
        lib.cudanet_end.restype = i32
        lib.cudanet_fingerprint.argtypes = [vp, cp, i32]
        lib.cudanet_fingerprint.restype = i32
        lib.cudanet_precision.argtypes = [vp, cp, i32]
        lib.cudanet_precision.restype = i32
        lib.cudanet_max_batch.argtypes = [vp]
        lib.cudanet_max_batch.restype = i32
        lib.cudanet_profile.argtypes = [vp, i32, i32, ctypes.POINTER(ctypes.c_double), i32, cp, i32]
        lib.cudanet_profile.restype = i32
        lib.cudanet_profile_names.argtypes = [cp, i32]
        lib.cudanet_profile_names.restype = i32
        lib.cudanet_destroy.argtypes = [vp]
        lib.cudanet_destroy.restype = None
        lib.cudanet_evaluate_device.argtypes = [vp, i32, i32] + [vp] * 10 + [cp, i32]
        lib.cudanet_evaluate_device.restype = i32
        lib.cudanet_check.argtypes = [vp, vp, cp, i32]
        lib.cudanet_check.restype = i32
        lib.cudanet_k_gemm.argtypes = [i32, i32, i32, vp, vp, vp, vp, i32, i32, i32, i32, vp, cp, i32]
        lib.cudanet_k_gemm.restype = i32
        lib.cudanet_k_gemm_noalloc.argtypes = [i32, i32, i32, vp, vp, vp, vp, i32, i32, i32, i32, vp, cp, i32]
        lib.cudanet_k_gemm_noalloc.restype = i32
        lib.cudanet_k_gemm_resln.argtypes = [i32, vp, vp, vp, vp, vp, vp, vp, i32, i32, i32, vp, cp, i32]
        lib.cudanet_k_gemm_resln.restype = i32
        lib.cudanet_k_attention.argtypes = [i32, vp, vp, i32, i32, i32, vp, cp, i32]
        lib.cudanet_k_attention.restype = i32
        lib.cudanet_k_attention_tc.argtypes = [i32, vp, vp, i32, i32, i32, vp, cp, i32]
        lib.cudanet_k_attention_tc.restype = i32
        lib.cudanet_k_attention_kernel.argtypes = [i32, i32, i32, vp, vp, i32, i32, i32, ctypes.c_float, vp, cp, i32]
        lib.cudanet_k_attention_kernel.restype = i32
        lib.cudanet_k_attention_cls.argtypes = [i32, vp, vp, i32, i32, i32, vp, cp, i32]
        lib.cudanet_k_attention_cls.restype = i32
        lib.cudanet_k_layernorm.argtypes = [i32, vp, vp, vp, vp, i32, i32, i32, vp, cp, i32]
        lib.cudanet_k_layernorm.restype = i32
        f32 = ctypes.c_float
        lib.cudanet_calibrate.argtypes = [vp, i32, vp, vp, vp, vp, vp, i32, cp, i32]
        lib.cudanet_calibrate.restype = i32
        lib.cudanet_k_gemm_f8.argtypes = [i32, i32, vp, vp, vp, vp, f32, vp, i32, i32, i32, i32, vp, cp, i32]
        lib.cudanet_k_gemm_f8.restype = i32
        lib.cudanet_k_attention_f8.argtypes = [vp, vp, i32, i32, i32, f32, vp, cp, i32]
        lib.cudanet_k_attention_f8.restype = i32
        lib.cudanet_k_layernorm_f8.argtypes = [i32, vp, vp, vp, vp, i32, i32, i32, f32, vp, cp, i32]
        lib.cudanet_k_layernorm_f8.restype = i32
        lib.cudanet_evaluate_keys.argtypes = [vp, i32, i32] + [vp] * 8 + [cp, i32]
        lib.cudanet_evaluate_keys.restype = i32
        lib.cudanet_begin_keys.argtypes = [vp, i32, i32] + [vp] * 5 + [cp, i32]
        lib.cudanet_begin_keys.restype = i32
        lib.cudanet_encode_keys.argtypes = [vp, vp, vp, i32, vp, vp, vp, vp, vp, cp, i32]
        lib.cudanet_encode_keys.restype = i32
        _libs[path] = lib
        return lib


def _as_c(value, dtype, shape, name):
    """`value` as a C-ordered array of `dtype` that the library can read in place; numpy makes a new array only
    when the dtype or the memory order has to change (a bool mask is reinterpreted as bytes, never copied).
    ValueError names the argument when its shape is not `shape`."""
    arr = np.asarray(value)
    if arr.dtype == np.bool_ and dtype is np.uint8:
        arr = arr.view(np.uint8)
    arr = np.require(np.atleast_1d(arr), dtype=dtype, requirements="C")
    if arr.shape == shape:
        return arr
    raise ValueError(f"{name}: shape {arr.shape}, expected {shape}")


# The six position inputs MCTS._prepare hands the evaluator: name, element type and shape for (B, wide).
_POSITION_INPUTS = (("ids", np.int64, lambda B, w: (B, 64)), ("cast", np.float32, lambda B, w: (B, 4)),
                    ("hm", np.int64, lambda B, w: (B,)), ("ep", np.int64, lambda B, w: (B,)),
                    ("I", np.int64, lambda B, w: (B, w)), ("M", np.uint8, lambda B, w: (B, w)))
# The key-fed form: transposition keys instead of the encoded board.
_KEY_INPUTS = (("keys", np.uint64, lambda B, w: (B, 10)), ("ep_sq", np.int64, lambda B, w: (B,)),
               ("clock", np.int64, lambda B, w: (B,)), ("I", np.int64, lambda B, w: (B, w)),
               ("M", np.uint8, lambda B, w: (B, w)))


def _p(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def _msg(err):
    return err.value.decode("utf-8", "replace")


class CudaNet:
    """One evaluator handle: the weights on one B200, a CUDA graph per batch size. One call at a time."""

    def __init__(self, weights_path, device=0, dll=None):
        self.path, self.device, self.dll = os.path.abspath(weights_path), int(device), dll_path(dll)
        self._lib, self._lock, self._h = load(self.dll), threading.Lock(), None
        reason = ctypes.create_string_buffer(ERR_LEN)
        handle = self._lib.cudanet_create(self.path.encode("utf-8"), self.device, reason, ERR_LEN)
        if handle:
            self._h = ctypes.c_void_p(handle)
            self.max_batch = int(self._lib.cudanet_max_batch(self._h))
            return
        raise RuntimeError(f"cudanet_create({self.path}): {_msg(reason)}")

    def _batch_dims(self, I):
        """(B, wide) of a call, from the move-index matrix I, after the checks every entry point makes."""
        if self._h is None:
            raise RuntimeError("CudaNet is closed")
        shape = np.shape(I)
        if len(shape) != 2:
            raise ValueError(f"I: shape {shape}, expected (B, wide)")
        B, wide = shape
        if B < 1 or B > self.max_batch:
            raise ValueError(f"batch {B}: cudanet takes 1 to {self.max_batch} (env MAYFLY_CUDANET_MAX_BATCH)")
        if wide < 1:
            raise ValueError("wide must be at least 1")
        return B, wide

    def _convert(self, spec, values):
        B, wide = self._batch_dims(values[-2])
        return (B, wide) + tuple(_as_c(v, dt, shape(B, wide), name) for (name, dt, shape), v in zip(spec, values))

    def _inputs(self, ids, cast, hm, ep, I, M):
        return self._convert(_POSITION_INPUTS, (ids, cast, hm, ep, I, M))

    def evaluate(self, ids, cast, hm, ep, I, M):
        """One batch. Returns (pol (B, wide), val (B,), qv (B, wide)) float32."""
        B, wide, ids, cast, hm, ep, I, M = self._inputs(ids, cast, hm, ep, I, M)
        pol = np.zeros((B, wide), np.float32)
        val = np.zeros(B, np.float32)
        qv = np.zeros((B, wide), np.float32)
        err = ctypes.create_string_buffer(ERR_LEN)
        with self._lock:
            rc = self._lib.cudanet_evaluate(self._h, B, wide, _p(ids), _p(cast), _p(hm), _p(ep), _p(I), _p(M),
                                            _p(pol), _p(val), _p(qv), err, ERR_LEN)
        if rc != 0:
            raise RuntimeError(f"cudanet_evaluate: {_msg(err)}")
        return pol, val, qv

    def _key_inputs(self, keys, ep_sq, clock, I, M):
        return self._convert(_KEY_INPUTS, (keys, ep_sq, clock, I, M))

    def evaluate_keys(self, keys, ep_sq, clock, I, M):
        """evaluate from transposition keys: keys (B, 10) uint64 = Board._transposition_key()[0:10] (turn and
        castling rights as integers), ep_sq (B,) the key's en passant square or -1 for None, clock (B,) the
        halfmove clocks. The GPU encodes them exactly as mayfly/chess/encode.py encode_keys does."""
        B, wide, keys, ep_sq, clock, I, M = self._key_inputs(keys, ep_sq, clock, I, M)
        pol = np.zeros((B, wide), np.float32)
        val = np.zeros(B, np.float32)
        qv = np.zeros((B, wide), np.float32)
        err = ctypes.create_string_buffer(ERR_LEN)
        with self._lock:
            rc = self._lib.cudanet_evaluate_keys(self._h, B, wide, _p(keys), _p(ep_sq), _p(clock), _p(I), _p(M),
                                                 _p(pol), _p(val), _p(qv), err, ERR_LEN)
        if rc != 0:
            raise RuntimeError(f"cudanet_evaluate_keys: {_msg(err)}")
        return pol, val, qv

    def begin_keys(self, keys, ep_sq, clock, I, M):
        """begin from transposition keys (see evaluate_keys); end() returns the outputs."""
        B, wide, keys, ep_sq, clock, I, M = self._key_inputs(keys, ep_sq, clock, I, M)
        err = ctypes.create_string_buffer(ERR_LEN)
        with self._lock:
            rc = self._lib.cudanet_begin_keys(self._h, B, wide, _p(keys), _p(ep_sq), _p(clock), _p(I), _p(M), err,
                                              ERR_LEN)
            if rc == 0:
                self._fly = getattr(self, "_fly", []) + [(B, wide)]
        if rc != 0:
            raise RuntimeError(f"cudanet_begin_keys: {_msg(err)}")

    def evaluate_logits(self, ids, cast, hm, ep, I, M):
        """evaluate, plus the full logits (B, 2 * 4162) float32: policy, then qvalue."""
        B, wide, ids, cast, hm, ep, I, M = self._inputs(ids, cast, hm, ep, I, M)
        pol = np.zeros((B, wide), np.float32)
        val = np.zeros(B, np.float32)
        qv = np.zeros((B, wide), np.float32)
        logits = np.zeros((B, 2 * N_MOVES), np.float32)
        err = ctypes.create_string_buffer(ERR_LEN)
        with self._lock:
            rc = self._lib.cudanet_evaluate_logits(self._h, B, wide, _p(ids), _p(cast), _p(hm), _p(ep), _p(I),
                                                   _p(M), _p(pol), _p(val), _p(qv), _p(logits), err, ERR_LEN)
        if rc != 0:
            raise RuntimeError(f"cudanet_evaluate_logits: {_msg(err)}")
        return pol, val, qv, logits

    def begin(self, ids, cast, hm, ep, I, M):
        """Queue one batch (at most two in flight); end() returns the oldest one's outputs."""
        B, wide, ids, cast, hm, ep, I, M = self._inputs(ids, cast, hm, ep, I, M)
        err = ctypes.create_string_buffer(ERR_LEN)
        with self._lock:
            rc = self._lib.cudanet_begin(self._h, B, wide, _p(ids), _p(cast), _p(hm), _p(ep), _p(I), _p(M), err,
                                         ERR_LEN)
            if rc == 0:
                self._fly = getattr(self, "_fly", []) + [(B, wide)]
        if rc != 0:
            raise RuntimeError(f"cudanet_begin: {_msg(err)}")

    def end(self):
        fly = getattr(self, "_fly", [])
        if not fly:
            raise RuntimeError("cudanet_end: no batch in flight")
        B, wide = fly[0]
        pol = np.zeros((B, wide), np.float32)
        val = np.zeros(B, np.float32)
        qv = np.zeros((B, wide), np.float32)
        err = ctypes.create_string_buffer(ERR_LEN)
        with self._lock:
            self._fly = fly[1:]
            rc = self._lib.cudanet_end(self._h, _p(pol), _p(val), _p(qv), err, ERR_LEN)
        if rc != 0:
            raise RuntimeError(f"cudanet_end: {_msg(err)}")
        return pol, val, qv

    def evaluate_device(self, ids, cast, hm, ep, I, M, pol, val, qv, stream=None):
        """One batch on torch CUDA tensors of the handle's device (outputs preallocated float32), queued on
        `stream` (a torch.cuda.Stream, default the current stream) without waiting."""
        import torch
        if self._h is None:
            raise RuntimeError("CudaNet is closed")
        B, wide = I.shape
        for name, t, dt in (("ids", ids, torch.int64), ("cast", cast, torch.float32), ("hm", hm, torch.int64),
                            ("ep", ep, torch.int64), ("I", I, torch.int64), ("M", M, torch.uint8),
                            ("pol", pol, torch.float32), ("val", val, torch.float32), ("qv", qv, torch.float32)):
            if not t.is_cuda or t.dtype != dt or not t.is_contiguous():
                raise ValueError(f"{name}: needs a contiguous CUDA {dt} tensor")
        s = stream if stream is not None else torch.cuda.current_stream()
        err = ctypes.create_string_buffer(ERR_LEN)
        with self._lock:
            rc = self._lib.cudanet_evaluate_device(self._h, B, wide, ids.data_ptr(), cast.data_ptr(),
                                                   hm.data_ptr(), ep.data_ptr(), I.data_ptr(), M.data_ptr(),
                                                   pol.data_ptr(), val.data_ptr(), qv.data_ptr(),
                                                   ctypes.c_void_p(s.cuda_stream), err, ERR_LEN)
        if rc != 0:
            raise RuntimeError(f"cudanet_evaluate_device: {_msg(err)}")

    def check(self, stream=None):
        """Wait for the handle's work (and `stream`) and raise if a device-side wait failed."""
        err = ctypes.create_string_buffer(ERR_LEN)
        sp = ctypes.c_void_p(stream.cuda_stream) if stream is not None else None
        with self._lock:
            rc = self._lib.cudanet_check(self._h, sp, err, ERR_LEN)
        if rc != 0:
            raise RuntimeError(f"cudanet_check: {_msg(err)}")

    def fingerprint(self):
        """The weight file's fingerprint, as mcts_cpp.fingerprint computes it for the checkpoint."""
        if self._h is None:
            raise RuntimeError("CudaNet is closed")
        buf = ctypes.create_string_buffer(256)
        if self._lib.cudanet_fingerprint(self._h, buf, len(buf)) < 0:
            raise RuntimeError("cudanet_fingerprint failed")
        return buf.value.decode("utf-8", "replace")

    def calibrate(self, ids, cast, hm, ep):
        """Runs the handle's 16-bit pass on these positions and returns max |.| of each layer's four product
        inputs (qkv, out, ff1, ff2) as float32 (layers, 4)."""
        if self._h is None:
            raise RuntimeError("CudaNet is closed")
        B, _ = self._batch_dims(np.empty((np.shape(ids)[0], 1)))
        ids, cast, hm, ep = (_as_c(v, dt, shape(B, 1), name)
                             for (name, dt, shape), v in zip(_POSITION_INPUTS[:4], (ids, cast, hm, ep)))
        out = np.zeros(4 * 256, np.float32)
        err = ctypes.create_string_buffer(ERR_LEN)
        with self._lock:
            k = self._lib.cudanet_calibrate(self._h, B, _p(ids), _p(cast), _p(hm), _p(ep), _p(out), out.size, err,
                                            ERR_LEN)
        if k < 0:
            raise RuntimeError(f"cudanet_calibrate: {_msg(err)}")
        return out[:k].reshape(-1, 4).copy()

    def precision(self):
        buf = ctypes.create_string_buffer(32)
        if self._lib.cudanet_precision(self._h, buf, len(buf)) < 0:
            raise RuntimeError("cudanet_precision failed")
        return buf.value.decode()

    def profile(self, B, reps=20):
        """Milliseconds a pass by step at batch B (an empty board, eager, an event after each step), the mean of
        reps passes, and last graph_pass, the whole pass as a CUDA graph. A dict in pass order."""
        if self._h is None:
            raise RuntimeError("CudaNet is closed")
        buf = ctypes.create_string_buffer(512)
        self._lib.cudanet_profile_names(buf, len(buf))
        names = buf.value.decode("utf-8").split(",")
        ms = (ctypes.c_double * len(names))()
        err = ctypes.create_string_buffer(ERR_LEN)
        with self._lock:
            k = self._lib.cudanet_profile(self._h, int(B), int(reps), ms, len(names), err, ERR_LEN)
        if k < 0:
            raise RuntimeError(f"cudanet_profile: {_msg(err)}")
        return dict(zip(names[:k], list(ms)[:k]))

    def close(self):
        if getattr(self, "_h", None) is not None:
            self._lib.cudanet_destroy(self._h)
            self._h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


# ------------------------------------------------------------------------------------------------ kernels
def _dtype_code(t):
    import torch
    if t.dtype == torch.float16:
        return 0
    if t.dtype == torch.bfloat16:
        return 1
    raise ValueError(f"16-bit float tensors only, got {t.dtype}")


def _stream():
    import torch
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def encode_keys_device(keys, ep_sq, clock, dll=None):
    """The GPU batch encoder on torch CUDA tensors: keys (B, 10) int64/uint64 words, ep_sq (B,) int64 (-1 for
    None), clock (B,) int64, on the current stream. Returns (ids (B, 64) int64, cast (B, 4) float32, hm (B,)
    int64, ep (B,) int64), encode.py encode_keys' values."""
    import torch
    lib = load(dll)
    B = keys.shape[0]
    for name, t in (("keys", keys), ("ep_sq", ep_sq), ("clock", clock)):
        if not t.is_cuda or t.element_size() != 8 or not t.is_contiguous():
            raise ValueError(f"{name}: needs a contiguous CUDA tensor of 64-bit words")
    if tuple(keys.shape) != (B, 10) or tuple(ep_sq.shape) != (B,) or tuple(clock.shape) != (B,):
        raise ValueError("keys (B, 10), ep_sq (B,), clock (B,)")
    dev = keys.device
    ids = torch.empty(B, 64, dtype=torch.int64, device=dev)
    cast = torch.empty(B, 4, dtype=torch.float32, device=dev)
    hm = torch.empty(B, dtype=torch.int64, device=dev)
    ep = torch.empty(B, dtype=torch.int64, device=dev)
    err = ctypes.create_string_buffer(ERR_LEN)
    rc = lib.cudanet_encode_keys(keys.data_ptr(), ep_sq.data_ptr(), clock.data_ptr(), B, ids.data_ptr(),
                                 cast.data_ptr(), hm.data_ptr(), ep.data_ptr(), _stream(), err, ERR_LEN)
    if rc != 0:
        raise RuntimeError(f"cudanet_encode_keys: {_msg(err)}")
    return ids, cast, hm, ep


def keys_from_tuples(keys):
    """Board._transposition_key() tuples (pawns .. castling rights, en passant square or None) as the arrays
    the key entry points take: (keys (B, 10) uint64, ep_sq (B,) int64 with -1 for None)."""
    B = len(keys)
    K = np.array([[int(k[j]) for j in range(10)] for k in keys], dtype=np.uint64).reshape(B, 10)
    ep = np.array([-1 if k[10] is None else int(k[10]) for k in keys], dtype=np.int64)
    return K, ep


def encode_keys(keys, hms, device=0, dll=None):
    """mayfly/chess/encode.py:73-100 encode_keys(keys, hms) with the same arguments and results (numpy ids
    (B, 64) int64, cast (B, 4) float32, hm (B,) int64, ep (B,) int64), computed by the GPU encoder."""
    import torch
    K, ep_sq = keys_from_tuples(keys)
    clock = np.asarray(hms, np.int64).reshape(len(keys))
    with torch.cuda.device(device):
        t = [torch.from_numpy(a.view(np.int64) if a.dtype == np.uint64 else a).cuda() for a in (K, ep_sq, clock)]
        out = encode_keys_device(*t, dll=dll)
        torch.cuda.current_stream().synchronize()
    return tuple(o.cpu().numpy() for o in out)


def k_gemm(A, W, bias, C, epi, bn=0, dll=None):
    """C = A W^T + epilogue on the tensor cores (epi 0 bias, 1 bias+GELU, 2 C += (f32), 3 f32 out)."""
    lib = load(dll)
    M, K = A.shape
    N = W.shape[0]
    err = ctypes.create_string_buffer(ERR_LEN)
    rc = lib.cudanet_k_gemm(_dtype_code(A), int(epi), int(bn), A.data_ptr(), W.data_ptr(), bias.data_ptr(),
                            C.data_ptr(), M, N, K, C.stride(0), _stream(), err, ERR_LEN)
    if rc != 0:
        raise RuntimeError(f"cudanet_k_gemm: {_msg(err)}")
    return C


def k_gemm_noalloc(A, W, bias, C, epi, bn=0, dll=None):
    """k_gemm without any device allocation: for callers that cannot call cudaMalloc (their GPU memory is
    reserved up front, or they must not stall in-flight work on an allocation). Its scratch is a static device
    array shared by every call; calls that overlap on the GPU race on it."""
    lib = load(dll)
    M, K = A.shape
    N = W.shape[0]
    err = ctypes.create_string_buffer(ERR_LEN)
    rc = lib.cudanet_k_gemm_noalloc(_dtype_code(A), int(epi), int(bn), A.data_ptr(), W.data_ptr(), bias.data_ptr(),
                                    C.data_ptr(), M, N, K, C.stride(0), _stream(), err, ERR_LEN)
    if rc != 0:
        raise RuntimeError(f"cudanet_k_gemm_noalloc: {_msg(err)}")
    return C


def k_gemm_resln(A, W, bias, X, g, b, H, dll=None):
    """X += A W^T + bias (f32, in place), then H = LayerNorm(X) * g + b (16-bit), in one fused kernel."""
    lib = load(dll)
    M, K = A.shape
    N = W.shape[0]
    err = ctypes.create_string_buffer(ERR_LEN)
    rc = lib.cudanet_k_gemm_resln(_dtype_code(A), A.data_ptr(), W.data_ptr(), bias.data_ptr(), X.data_ptr(),
                                  g.data_ptr(), b.data_ptr(), H.data_ptr(), M, N, K, _stream(), err, ERR_LEN)
    if rc != 0:
        raise RuntimeError(f"cudanet_k_gemm_resln: {_msg(err)}")
    return X, H


def k_attention(qkv, att, B, d, heads, dll=None):
    lib = load(dll)
    err = ctypes.create_string_buffer(ERR_LEN)
    rc = lib.cudanet_k_attention(_dtype_code(qkv), qkv.data_ptr(), att.data_ptr(), B, d, heads, _stream(), err,
                                 ERR_LEN)
    if rc != 0:
        raise RuntimeError(f"cudanet_k_attention: {_msg(err)}")
    return att


def k_attention_kernel(qkv, att, B, d, heads, kernel, mul=1.0, dll=None):
    """One attention launch on a chosen kernel (0 mma.sync, 1 two-group, 4 four-group tensor-memory, -1 the
    evaluator's choice); att uint8 gets e4m3 of att * mul (bf16 qkv), else att in qkv's type."""
    import torch
    lib = load(dll)
    err = ctypes.create_string_buffer(ERR_LEN)
    rc = lib.cudanet_k_attention_kernel(_dtype_code(qkv), 1 if att.dtype == torch.uint8 else 0, int(kernel),
                                        qkv.data_ptr(), att.data_ptr(), B, d, heads, float(mul), _stream(), err,
                                        ERR_LEN)
    if rc != 0:
        raise RuntimeError(f"cudanet_k_attention_kernel: {_msg(err)}")
    return att


def k_attention_tc(qkv, att, B, d, heads, dll=None):
    """k_attention on the tensor-memory (tcgen05) kernel, head width 64."""
    lib = load(dll)
    err = ctypes.create_string_buffer(ERR_LEN)
    rc = lib.cudanet_k_attention_tc(_dtype_code(qkv), qkv.data_ptr(), att.data_ptr(), B, d, heads, _stream(), err,
                                    ERR_LEN)
    if rc != 0:
        raise RuntimeError(f"cudanet_k_attention_tc: {_msg(err)}")
    return att


def k_attention_cls(qkv, att, B, d, heads, dll=None):
    """att [B, d] = attention of each board's CLS query (token 0) over its 65 tokens."""
    lib = load(dll)
    err = ctypes.create_string_buffer(ERR_LEN)
    rc = lib.cudanet_k_attention_cls(_dtype_code(qkv), qkv.data_ptr(), att.data_ptr(), B, d, heads, _stream(), err,
                                     ERR_LEN)
    if rc != 0:
        raise RuntimeError(f"cudanet_k_attention_cls: {_msg(err)}")
    return att


def k_layernorm(x, g, b, h, n, d, row_stride=1, dll=None):
    lib = load(dll)
    err = ctypes.create_string_buffer(ERR_LEN)
    rc = lib.cudanet_k_layernorm(_dtype_code(h), x.data_ptr(), g.data_ptr(), b.data_ptr(), h.data_ptr(), n, d,
                                 row_stride, _stream(), err, ERR_LEN)
    if rc != 0:
        raise RuntimeError(f"cudanet_k_layernorm: {_msg(err)}")
    return h


# ------------------------------------------------------------------------------------------------ FP8 kernels
def _e4m3(t, name):
    import torch
    if t.dtype not in (torch.float8_e4m3fn, torch.uint8):
        raise ValueError(f"{name}: e4m3 bytes (torch.float8_e4m3fn or uint8) only, got {t.dtype}")


def k_gemm_f8(A, W, colscale, bias, C, epi, out_scale_inv=1.0, bn=0, dll=None):
    """C = epilogue(A W^T * colscale + bias) with e4m3 A and W (epi 0 bf16 out, 2 C += (f32), 3 f32 out,
    4 e4m3 out of gelu(.) * out_scale_inv, 5 C += (bf16))."""
    _e4m3(A, "A")
    _e4m3(W, "W")
    lib = load(dll)
    M, K = A.shape
    N = W.shape[0]
    err = ctypes.create_string_buffer(ERR_LEN)
    rc = lib.cudanet_k_gemm_f8(int(epi), int(bn), A.data_ptr(), W.data_ptr(), colscale.data_ptr(), bias.data_ptr(),
                               float(out_scale_inv), C.data_ptr(), M, N, K, C.stride(0), _stream(), err, ERR_LEN)
    if rc != 0:
        raise RuntimeError(f"cudanet_k_gemm_f8: {_msg(err)}")
    return C


def k_attention_f8(qkv, att, B, d, heads, mul, dll=None):
    """att (e4m3) = e4m3(attention(qkv) * mul), qkv bf16."""
    _e4m3(att, "att")
    lib = load(dll)
    err = ctypes.create_string_buffer(ERR_LEN)
    rc = lib.cudanet_k_attention_f8(qkv.data_ptr(), att.data_ptr(), B, d, heads, float(mul), _stream(), err, ERR_LEN)
    if rc != 0:
        raise RuntimeError(f"cudanet_k_attention_f8: {_msg(err)}")
    return att


def k_layernorm_f8(x, g, b, h, n, d, mul, row_stride=1, dll=None):
    """h (e4m3) = e4m3(LayerNorm(x) * mul), x float32 or bfloat16."""
    import torch
    _e4m3(h, "h")
    if x.dtype not in (torch.float32, torch.bfloat16):
        raise ValueError(f"x: float32 or bfloat16 only, got {x.dtype}")
    lib = load(dll)
    err = ctypes.create_string_buffer(ERR_LEN)
    rc = lib.cudanet_k_layernorm_f8(int(x.dtype == torch.bfloat16), x.data_ptr(), g.data_ptr(), b.data_ptr(),
                                    h.data_ptr(), n, d, row_stride, float(mul), _stream(), err, ERR_LEN)
    if rc != 0:
        raise RuntimeError(f"cudanet_k_layernorm_f8: {_msg(err)}")
    return h
