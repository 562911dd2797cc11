"""ctypes binding of libnn_b200.so -- the Python mirror of COpenCLMy.

`Context` plays the role of the reference's COpenCLMy object
(Experts/NeuroNet_DNG/NeuroNet_Declarations.mqh:359-513): int buffer handles,
kernels created by id and NeuroNet.cl name, persistent positional arguments
and `execute(id, global, local)`.  Every failing call raises `NNError` with
the library's message; there is no fallback path -- a missing or unloadable
library is an error.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libnn_b200.so")

# ENUM_ACTIVATION (NeuroNet_Definitions.mqh:3650-3669) and ENUM_OPTIMIZATION (3671-3685)
NONE, TANH, SIGMOID, LRELU, SOFTPLUS, GELU, MINUS_SOFTPLUS, ELU = -1, 0, 1, 2, 3, 4, 5, 6
SGD, ADAM, LS, ADAM_MINI = 0, 1, 2, 3

# NeuroNet.cl kernel signatures: one char per positional argument (p buffer, i int, f float).
SIGNATURES = {
    "FeedForward": "pppiipi", "CalcOutputGradient": "pppif", "CalcHiddenGradient": "ppppii",
    "UpdateWeightsMomentum": "ppppiff", "UpdateWeightsAdam": "pppppifff",
    "UpdateWeightsAdamMini": "pppppfff", "UpdateWeightsConvAdamMini": "pppppifffi",
    "MatMult": "pppiiiiipi", "MatMultGrad": "pppppiiiiiii",
    "FQF_Cosine": "pp", "FQF_Output": "pppi", "FQF_OutputGradient": "ppppp", "FQF_QuantileGradient": "ppppp",
    "FQF_CosineGradient": "ppp", "FQF_FractionGradient": "pppi",
    "FQF_CosineGradientSRM": "ppp", "FQF_DistributionTargetGradient": "ppppfff",
    "FQF_MonotoneRearrange": "pppppp", "FQF_RearrangeGradient": "ppppp", "FQF_SRMForward": "pppiff",
    "FQF_SRMGradient": "pppppiff", "SAC_AlphaLogProbs": "ppppppii",
    "SAC_AlphaGradients": "ppppi",
    "SAC_OutputGradient": "ppppppii", "SAC_CalcLogProbs": "pppppii",
    "MHFlashAttention": "ppppiii", "MHFlashAttentionGrad": "pppppppiiii", "NormalizeWeights": "pi",
    "Activation": "ppi", "DeActivation": "pppi", "SoftUpdate": "ppf", "SoftUpdateAdam": "ppppfff",
    "FeedForwardConv": "pppiiiii", "CalcHiddenGradientConv": "ppppiiiiii",
    "UpdateWeightsConvAdam": "pppppifffiii", "UpdateWeightsConvMomentum": "ppppiffiii",
    "MHAttentionScore": "ppii", "MHAttentionOut": "pppi", "MHAttentionInsideGradients": "pppp",
    "SumMatrix": "pppifiiipi", "Normalize": "pi", "SoftMax_FeedForward": "pp",
    "SoftMax_HiddenGradient": "ppp", "SoftMax_OutputGradient": "ppp", "Transpose": "pp",
    "ConcatenateBuffers": "pipipipip", "DeconcatenateBuffers": "pipipipip",
    "RevInFeedForward": "pppii", "RevInHiddenGraddient": "ppppiii",
    "BatchFeedForward": "pppiiii", "CalcHiddenGradientBatch": "ppppiii",
    "UpdateBatchOptionsMomentum": "ppff", "UpdateBatchOptionsAdam": "ppfff",
    "LSTM_FeedForward": "pipppp", "LSTM_ConcatenatedGradient": "pppp",
    "LSTM_HiddenGradient": "pppppppii", "LSTM_UpdateWeightsAdam": "ppppfff",
    "Concat_FeedForward": "ppppiii", "Concat_HiddenGradient": "ppppppiiiii",
    "Concat_UpdateWeightsMomentum": "pppppiiff", "Concat_UpdateWeightsAdam": "ppppppiifff",
    "SACGaussianPolicy": "ppppi", "SACTargetValue": "ppppppff", "SACPolicyGradient": "ppppppppif",
    "MH2AttentionOut": "ppppiii", "MH2AttentionInsideGradients": "ppppppii",
    "AttentionScore": "pppii", "AttentionOut": "pppp", "AttentionInsideGradients": "pppppppp",
    "Dropout": "pppi", "PatchCreate": "pppiiii", "PatchHiddenGradient": "ppppiiiii",
    "PatchUpdateWeightsAdam": "pppppifffi", "FQF_Sample": "pppp",
}


class NNError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"[{status}] {message}")
        self.status = status


_LIB = None


def load_library(path: str = LIB_PATH) -> ctypes.CDLL:
    """Load libnn_b200.so once; raises if it is missing (no fallback)."""
    global _LIB
    if _LIB is not None:
        return _LIB
    if not os.path.exists(path):
        raise NNError(-1, f"{path} is missing: build it with `python -m nn_in_trading_b200.build`")
    lib = ctypes.CDLL(path)
    c_int, c_ll, c_f, c_p = ctypes.c_int, ctypes.c_longlong, ctypes.c_float, ctypes.c_void_p
    u32p = ctypes.POINTER(ctypes.c_uint)
    sig = {
        "nn_init": ([c_int, c_int], c_int), "nn_shutdown": ([], c_int),
        "nn_last_error": ([ctypes.c_char_p, c_int], c_int), "nn_max_local_size": ([c_int], c_int),
        "nn_finish": ([c_int], c_int), "nn_stream": ([], c_p),
        "nn_buffer_create": ([c_ll], c_int), "nn_buffer_free": ([c_int], c_int),
        "nn_buffer_write": ([c_int, c_p, c_ll, c_ll], c_int), "nn_buffer_read": ([c_int, c_p, c_ll, c_ll], c_int),
        "nn_buffer_write_ex": ([c_int, c_p, c_ll, c_ll, c_ll], c_int),
        "nn_buffer_read_ex": ([c_int, c_p, c_ll, c_ll, c_ll], c_int),
        "nn_buffer_fill": ([c_int, c_f, c_ll, c_ll], c_int),
        "nn_buffer_copy": ([c_int, c_ll, c_int, c_ll, c_ll], c_int),
        "nn_buffer_write_async": ([c_int, c_p, c_ll, c_ll], c_int),
        "nn_buffer_read_async": ([c_int, c_p, c_ll, c_ll], c_int), "nn_transfer_wait": ([c_int], c_int),
        "nn_buffer_bytes": ([c_int], c_ll), "nn_buffer_device_ptr": ([c_int], c_p),
        "nn_kernel_create": ([c_int, ctypes.c_char_p], c_int), "nn_kernel_free": ([c_int], c_int),
        "nn_set_arg_buffer": ([c_int, c_int, c_int], c_int), "nn_set_arg_int": ([c_int, c_int, c_int], c_int),
        "nn_set_arg_float": ([c_int, c_int, c_f], c_int), "nn_set_batch": ([c_int, c_int], c_int),
        "nn_execute": ([c_int, c_int, u32p, u32p, u32p], c_int), "nn_launch_count": ([], c_ll),
        "nn_cmdlist_begin": ([], c_int), "nn_cmdlist_end": ([], c_int), "nn_cmdlist_run": ([c_int], c_int),
        "nn_cmdlist_set_float": ([c_int, c_int, c_int, c_f], c_int),
        "nn_cmdlist_set_int": ([c_int, c_int, c_int, c_int], c_int),
        "nn_cmdlist_size": ([c_int], c_int), "nn_cmdlist_free": ([c_int], c_int),
        "nn_dp_unique_id": ([c_p], c_int), "nn_dp_init": ([c_int, c_int, c_p], c_int),
        "nn_dp_shutdown": ([], c_int), "nn_dp_allreduce": ([c_int, c_ll, c_ll, c_f], c_int),
        "nn_dp_update_begin": ([], c_int), "nn_dp_update_end": ([], c_int),
        "nn_update_weights_adam_fixed": ([c_p, c_p, c_p, c_p, c_p, c_int, c_int, c_int, c_f, c_f, c_f], c_int),
    }
    for name, (args, res) in sig.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = res
    _LIB = lib
    return lib


def _u32(values):
    if values is None:
        return None
    values = list(values)
    return (ctypes.c_uint * len(values))(*[int(v) for v in values])


class Context:
    """One library context on one CUDA device (COpenCLMy equivalent)."""

    def __init__(self, device: int = 0):
        self.lib = load_library()
        self._check(self.lib.nn_init(device, 0))
        self.device = device
        self._next_kernel = 1
        self.alive = True

    # -- errors -------------------------------------------------------------
    def last_error(self) -> str:
        buf = ctypes.create_string_buffer(1024)
        self.lib.nn_last_error(buf, 1024)
        return buf.value.decode(errors="replace")

    def _check(self, rc: int) -> int:
        if rc < 0:
            raise NNError(rc, self.last_error())
        return rc

    def close(self) -> None:
        if self.alive:
            self._check(self.lib.nn_shutdown())
            self.alive = False

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    # -- buffers ------------------------------------------------------------
    def buffer(self, count: int, fill: float | None = 0.0) -> int:
        """Create a buffer of `count` floats (zero-filled)."""
        h = self._check(self.lib.nn_buffer_create(max(int(count), 1) * 4))
        if fill not in (None, 0.0):
            self._check(self.lib.nn_buffer_fill(h, float(fill), 0, int(count)))
        return h

    def free(self, h: int) -> None:
        self._check(self.lib.nn_buffer_free(h))

    def write(self, h: int, data, offset: int = 0) -> None:
        a = np.ascontiguousarray(data, dtype=np.float32).reshape(-1)
        self._check(self.lib.nn_buffer_write(h, a.ctypes.data, int(offset), a.size))

    def read(self, h: int, count: int | None = None, offset: int = 0, out: np.ndarray | None = None) -> np.ndarray:
        if count is None:
            count = self.lib.nn_buffer_bytes(h) // 4 - offset
        if out is None:
            out = np.empty(int(count), dtype=np.float32)
        self._check(self.lib.nn_buffer_read(h, out.ctypes.data, int(offset), int(count)))
        return out

    def fill(self, h: int, value: float, count: int, offset: int = 0) -> None:
        self._check(self.lib.nn_buffer_fill(h, float(value), int(offset), int(count)))

    def copy(self, dst: int, src: int, count: int, dst_offset: int = 0, src_offset: int = 0) -> None:
        self._check(self.lib.nn_buffer_copy(dst, int(dst_offset), src, int(src_offset), int(count)))

    def nbytes(self, h: int) -> int:
        return self._check(self.lib.nn_buffer_bytes(h))

    def device_ptr(self, h: int) -> int:
        return self.lib.nn_buffer_device_ptr(h)

    # -- kernels ------------------------------------------------------------
    def kernel(self, name: str, kid: int | None = None) -> "Kernel":
        if kid is None:
            kid = self._next_kernel
            self._next_kernel += 1
        self._check(self.lib.nn_kernel_create(kid, name.encode()))
        return Kernel(self, kid, name)

    def execute(self, kid: int, global_size, local_size=None) -> None:
        g = list(global_size)
        self._check(self.lib.nn_execute(kid, len(g), None, _u32(g), _u32(local_size)))

    def finish(self, timeout_ms: int = 0) -> None:
        self._check(self.lib.nn_finish(int(timeout_ms)))

    def stream(self) -> int:
        return self.lib.nn_stream()

    def launch_count(self) -> int:
        return int(self.lib.nn_launch_count())

    # -- command lists --------------------------------------------------------
    def record_begin(self) -> None:
        self._check(self.lib.nn_cmdlist_begin())

    def record_end(self) -> int:
        return self._check(self.lib.nn_cmdlist_end())

    def run_list(self, lid: int) -> None:
        self._check(self.lib.nn_cmdlist_run(lid))

    def list_set_float(self, lid: int, pos: int, idx: int, value: float) -> None:
        self._check(self.lib.nn_cmdlist_set_float(lid, pos, idx, float(value)))

    def free_list(self, lid: int) -> None:
        self._check(self.lib.nn_cmdlist_free(lid))

    # -- data parallel --------------------------------------------------------
    def dp_unique_id(self) -> bytes:
        buf = (ctypes.c_ubyte * 128)()
        self._check(self.lib.nn_dp_unique_id(ctypes.addressof(buf)))
        return bytes(buf)

    def dp_init(self, rank: int, world: int, uid: bytes) -> None:
        buf = (ctypes.c_ubyte * 128).from_buffer_copy(uid)
        self._check(self.lib.nn_dp_init(rank, world, ctypes.addressof(buf)))

    def dp_shutdown(self) -> None:
        self._check(self.lib.nn_dp_shutdown())

    def dp_allreduce(self, h: int, count: int, scale: float = 1.0, offset: int = 0) -> None:
        self._check(self.lib.nn_dp_allreduce(h, int(offset), int(count), float(scale)))

    def dp_update_begin(self) -> None:
        self._check(self.lib.nn_dp_update_begin())

    def dp_update_end(self) -> None:
        self._check(self.lib.nn_dp_update_end())


class Kernel:
    """A kernel instance with persistent positional arguments (COpenCL kernel handle)."""

    def __init__(self, ctx: Context, kid: int, name: str):
        self.ctx, self.id, self.name = ctx, kid, name
        self.sig = SIGNATURES[name]
        self.values = {}  # last value bound to each argument index
        self.b = 1  # batch set with nn_set_batch

    def set(self, idx: int, value) -> "Kernel":
        t = self.sig[idx]
        lib = self.ctx.lib
        self.values[idx] = value
        if t == "p":
            self.ctx._check(lib.nn_set_arg_buffer(self.id, idx, int(value)))
        elif t == "f":
            self.ctx._check(lib.nn_set_arg_float(self.id, idx, float(value)))
        else:
            self.ctx._check(lib.nn_set_arg_int(self.id, idx, int(value)))
        return self

    def args(self, *values) -> "Kernel":
        for i, v in enumerate(values):
            if v is not None:
                self.set(i, v)
        return self

    def batch(self, b: int) -> "Kernel":
        self.ctx._check(self.ctx.lib.nn_set_batch(self.id, int(b)))
        self.b = int(b)
        return self

    def run(self, global_size, local_size=None) -> None:
        self.ctx.execute(self.id, global_size, local_size)
