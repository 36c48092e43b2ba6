"""ctypes binding of libm3cuda.so (include/m3_cuda.h).

The library exports the graph/session API of m3.c's include/m3.h, the
reference backend plug-in functions and the CUDA extensions.  This module
mirrors those C types and wraps the graph/session API in two small classes.
The wrappers only need the m3.h ABI, so `Graph(lib=...)`/`Session(lib=...)`
also drive any other library exporting the same API.

Loading fails loudly when libm3cuda.so is missing: there is no Python or CPU
fallback for the provider.
"""

from __future__ import annotations

import ctypes
import os
from typing import Iterable, Sequence

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIBRARY_PATH = os.path.join(HERE, "libm3cuda.so")

# include/m3.h:20-31
OK, INVALID_ARGUMENT, OUT_OF_RANGE, OVERFLOW, OUT_OF_MEMORY = 0, 1, 2, 3, 4
IO, INVALID_FORMAT, UNSUPPORTED, CANCELLED, INTERNAL = 5, 6, 7, 8, 9
# include/m3.h:45-50
F32, F16, BF16, I32 = 0, 1, 2, 3
# include/m3.h:52-73 and the CUDA extensions
OPS = dict(COPY=0, CAST=1, ADD=2, MUL=3, EMBEDDING=4, MATMUL=5, LINEAR=6,
           RMS_NORM=7, LAYER_NORM=8, ROPE=9, ATTENTION=10, GATED_SILU=11,
           SOFTMAX=12, TOP_K=13, CATEGORICAL=14, CONV1D=15,
           CONV_TRANSPOSE1D=16, NEAREST_RESIZE1D=17, SNAKE1D=18, TANH=19,
           ABS_MAX=64, CLAMP_UNIT=65, ROW_SUM=66)
# include/m3.h:80-91
PROVIDER_NEURAL_ENGINE, PROVIDER_METAL, PROVIDER_CPU, PROVIDER_CUDA = 0, 1, 2, 3
INPUT, CONSTANT, TEMPORARY, OUTPUT = 0, 1, 2, 3
VALUE_NONE = 0xFFFFFFFF
MAX_RANK = 8

NUMPY_OF = {F32: np.float32, F16: np.uint16, BF16: np.uint16, I32: np.int32}
ITEMSIZE = {F32: 4, F16: 2, BF16: 2, I32: 4}


class M3Error(ctypes.Structure):
    _fields_ = [("status", ctypes.c_int), ("message", ctypes.c_char * 256)]


class GraphValueDesc(ctypes.Structure):
    _fields_ = [("dtype", ctypes.c_int), ("rank", ctypes.c_uint8),
                ("shape", ctypes.c_uint64 * MAX_RANK), ("role", ctypes.c_int)]


class _Norm(ctypes.Structure):
    _fields_ = [("epsilon", ctypes.c_float)]


class _Rope(ctypes.Structure):
    _fields_ = [("position_offset", ctypes.c_uint64),
                ("rotary_dimension", ctypes.c_uint32), ("mode", ctypes.c_int)]


class _Attention(ctypes.Structure):
    _fields_ = [("scale", ctypes.c_float), ("causal_offset", ctypes.c_int64),
                ("causal", ctypes.c_bool)]


class _TopK(ctypes.Structure):
    _fields_ = [("k", ctypes.c_uint64)]


class _Convolution(ctypes.Structure):
    _fields_ = [(n, ctypes.c_uint64) for n in (
        "groups", "stride", "dilation", "pad_left", "pad_right",
        "output_padding")]


class _Resize(ctypes.Structure):
    _fields_ = [("output_length", ctypes.c_uint64)]


class _Parameters(ctypes.Union):
    _fields_ = [("norm", _Norm), ("rope", _Rope), ("attention", _Attention),
                ("top_k", _TopK), ("convolution", _Convolution),
                ("resize", _Resize)]


class NodeDesc(ctypes.Structure):
    _fields_ = [("kind", ctypes.c_int), ("inputs", ctypes.c_uint32 * 5),
                ("outputs", ctypes.c_uint32 * 2), ("parameters", _Parameters)]


class SessionOptions(ctypes.Structure):
    _fields_ = [("allow_neural_engine", ctypes.c_bool),
                ("allow_metal", ctypes.c_bool), ("allow_cpu", ctypes.c_bool)]


class PlanInfo(ctypes.Structure):
    _fields_ = [("value_count", ctypes.c_size_t),
                ("node_count", ctypes.c_size_t),
                ("storage_slot_count", ctypes.c_size_t),
                ("allocated_bytes", ctypes.c_size_t)]


class CudaSessionOptions(ctypes.Structure):
    _fields_ = [("device", ctypes.c_int), ("stream", ctypes.c_void_p),
                ("fuse", ctypes.c_bool), ("cuda_graphs", ctypes.c_bool)]


class ShardOptions(ctypes.Structure):
    """m3_cuda_shard_options: this rank's place in a graph split across
    `count` GPUs along `axis` (AXIS_AUTO: the library's choice); `id` is the
    communicator id (ShardId or None: no collective)."""

    AXIS_AUTO = -1

    def __init__(self, rank: int = 0, count: int = 1, axis: int = -1, id=None,
                 timeout_seconds: float = 120.0):
        super().__init__()
        self.rank = rank
        self.count = count
        self.axis = axis
        self._id = id
        self.id = ctypes.pointer(id) if id is not None else None
        self.timeout_seconds = timeout_seconds


class ShardId(ctypes.Structure):
    _fields_ = [("bytes", ctypes.c_ubyte * 128)]


ShardOptions._fields_ = [("rank", ctypes.c_int), ("count", ctypes.c_int),
                         ("axis", ctypes.c_int), ("id", ctypes.POINTER(ShardId)),
                         ("timeout_seconds", ctypes.c_double)]


class PlanReport(ctypes.Structure):
    _fields_ = [("launch_count", ctypes.c_size_t),
                ("fused_node_count", ctypes.c_size_t),
                ("shadow_bytes", ctypes.c_size_t),
                ("arena_bytes", ctypes.c_size_t)]


# src/m3_tensor.h:12-27
class TensorMetadata(ctypes.Structure):
    _fields_ = [("dtype", ctypes.c_int), ("rank", ctypes.c_uint8),
                ("shape", ctypes.c_uint64 * MAX_RANK),
                ("element_count", ctypes.c_size_t),
                ("byte_count", ctypes.c_size_t)]


class ShardSlab(ctypes.Structure):
    """m3_cuda_shard_slab: where one value's slab lies in the global tensor."""

    _fields_ = [("split", ctypes.c_bool), ("axis", ctypes.c_uint8),
                ("begin", ctypes.c_uint64), ("extent", ctypes.c_uint64),
                ("global_", TensorMetadata), ("local", TensorMetadata)]


class TensorView(ctypes.Structure):
    _fields_ = [("metadata", TensorMetadata), ("byte_offset", ctypes.c_size_t),
                ("byte_strides", ctypes.c_size_t * MAX_RANK),
                ("storage", ctypes.c_void_p)]


_VP = ctypes.POINTER(TensorView)


class _Unary(ctypes.Structure):
    _fields_ = [("input", _VP), ("output", _VP)]


class _Binary(ctypes.Structure):
    _fields_ = [("left", _VP), ("right", _VP), ("output", _VP)]


class _RmsNorm(ctypes.Structure):
    _fields_ = [("input", _VP), ("scale", _VP), ("output", _VP),
                ("epsilon", ctypes.c_float)]


class _LayerNorm(ctypes.Structure):
    _fields_ = [("input", _VP), ("scale", _VP), ("bias", _VP),
                ("output", _VP), ("epsilon", ctypes.c_float)]


class _TopKCommand(ctypes.Structure):
    _fields_ = [("logits", _VP), ("values", _VP), ("indices", _VP),
                ("k", ctypes.c_uint64)]


class _Snake(ctypes.Structure):
    _fields_ = [("input", _VP), ("alpha", _VP), ("output", _VP)]


class _Categorical(ctypes.Structure):
    _fields_ = [("probabilities", _VP), ("uniforms", _VP), ("output", _VP)]


class _ConvTranspose(ctypes.Structure):
    # the largest member of the reference union (src/m3_op.h:105-116)
    _fields_ = [("input", _VP), ("weight", _VP), ("bias", _VP),
                ("output", _VP)] + [(n, ctypes.c_uint64) for n in (
                    "groups", "stride", "dilation", "pad_left", "pad_right",
                    "output_padding")]


class _Descriptor(ctypes.Union):
    _fields_ = [("copy", _Unary), ("cast", _Unary), ("add", _Binary),
                ("mul", _Binary), ("rms_norm", _RmsNorm),
                ("layer_norm", _LayerNorm), ("gated_silu", _Binary),
                ("softmax", _Unary), ("top_k", _TopKCommand),
                ("snake1d", _Snake), ("tanh", _Unary),
                ("categorical", _Categorical),
                ("conv_transpose1d", _ConvTranspose)]


class Command(ctypes.Structure):
    _fields_ = [("kind", ctypes.c_int), ("descriptor", _Descriptor)]


STORAGE_DATA = ctypes.CFUNCTYPE(ctypes.c_void_p, ctypes.c_void_p)


class BackendOptions(ctypes.Structure):
    _fields_ = [("device", ctypes.c_int), ("storage_data", STORAGE_DATA),
                ("managed_memory", ctypes.c_bool)]


class M3Failure(RuntimeError):
    """A non-OK m3_status, with the library's message."""

    def __init__(self, status: int, message: str):
        super().__init__(f"status {status}: {message}")
        self.status = status
        self.message = message


_library = None

_SIGNATURES = {
    "m3_version": (ctypes.c_char_p, []),
    "m3_status_string": (ctypes.c_char_p, [ctypes.c_int]),
    "m3_graph_value_desc_init": (None, [ctypes.POINTER(GraphValueDesc),
                                        ctypes.c_int, ctypes.c_int,
                                        ctypes.c_uint8,
                                        ctypes.POINTER(ctypes.c_uint64)]),
    "m3_graph_node_desc_init": (None, [ctypes.POINTER(NodeDesc), ctypes.c_int]),
    "m3_session_options_init": (None, [ctypes.POINTER(SessionOptions)]),
    "m3_graph_create": (ctypes.c_int, [ctypes.POINTER(ctypes.c_void_p),
                                       ctypes.POINTER(M3Error)]),
    "m3_graph_free": (None, [ctypes.c_void_p]),
    "m3_graph_add_value": (ctypes.c_int, [ctypes.c_void_p,
                                          ctypes.POINTER(GraphValueDesc),
                                          ctypes.POINTER(ctypes.c_uint32),
                                          ctypes.POINTER(M3Error)]),
    "m3_graph_set_constant": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_uint32,
                                             ctypes.c_void_p, ctypes.c_size_t,
                                             ctypes.POINTER(M3Error)]),
    "m3_graph_add_inferred_value": (ctypes.c_int, [
        ctypes.c_void_p, ctypes.POINTER(NodeDesc), ctypes.c_size_t,
        ctypes.c_int, ctypes.c_int, ctypes.POINTER(ctypes.c_uint32),
        ctypes.POINTER(M3Error)]),
    "m3_graph_add_node": (ctypes.c_int, [ctypes.c_void_p,
                                         ctypes.POINTER(NodeDesc),
                                         ctypes.POINTER(M3Error)]),
    "m3_session_create": (ctypes.c_int, [ctypes.POINTER(ctypes.c_void_p),
                                         ctypes.c_void_p,
                                         ctypes.POINTER(SessionOptions),
                                         ctypes.POINTER(M3Error)]),
    "m3_session_free": (None, [ctypes.c_void_p]),
    "m3_session_write_input": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_uint32,
                                              ctypes.c_void_p, ctypes.c_size_t,
                                              ctypes.POINTER(M3Error)]),
    "m3_session_read_output": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_uint32,
                                              ctypes.c_void_p, ctypes.c_size_t,
                                              ctypes.POINTER(M3Error)]),
    "m3_session_run": (ctypes.c_int, [ctypes.c_void_p,
                                      ctypes.POINTER(M3Error)]),
    "m3_session_get_plan_info": (ctypes.c_int, [ctypes.c_void_p,
                                                ctypes.POINTER(PlanInfo),
                                                ctypes.POINTER(M3Error)]),
    "m3_session_get_node_provider": (ctypes.c_int, [
        ctypes.c_void_p, ctypes.c_size_t, ctypes.POINTER(ctypes.c_int),
        ctypes.POINTER(M3Error)]),
}

_CUDA_SIGNATURES = {
    "m3_cuda_session_options_init": (None, [ctypes.POINTER(CudaSessionOptions)]),
    "m3_cuda_session_create": (ctypes.c_int, [
        ctypes.POINTER(ctypes.c_void_p), ctypes.c_void_p,
        ctypes.POINTER(SessionOptions), ctypes.POINTER(CudaSessionOptions),
        ctypes.POINTER(M3Error)]),
    "m3_cuda_session_run_async": (ctypes.c_int, [ctypes.c_void_p,
                                                 ctypes.POINTER(M3Error)]),
    "m3_cuda_session_submit_host_async": (ctypes.c_int, [
        ctypes.c_void_p, ctypes.c_size_t, ctypes.POINTER(ctypes.c_uint32),
        ctypes.POINTER(ctypes.c_void_p), ctypes.c_size_t, ctypes.POINTER(ctypes.c_uint32),
        ctypes.POINTER(ctypes.c_void_p), ctypes.POINTER(M3Error)]),
    "m3_cuda_session_run_steps_async": (ctypes.c_int, [
        ctypes.c_void_p, ctypes.c_size_t, ctypes.c_uint32, ctypes.c_uint32,
        ctypes.POINTER(M3Error)]),
    "m3_cuda_session_synchronize": (ctypes.c_int, [ctypes.c_void_p,
                                                   ctypes.POINTER(M3Error)]),
    "m3_cuda_session_value_device_pointer": (ctypes.c_int, [
        ctypes.c_void_p, ctypes.c_uint32, ctypes.POINTER(ctypes.c_void_p),
        ctypes.POINTER(ctypes.c_size_t), ctypes.POINTER(M3Error)]),
    "m3_cuda_session_write_input_device": (ctypes.c_int, [
        ctypes.c_void_p, ctypes.c_uint32, ctypes.c_void_p, ctypes.c_size_t,
        ctypes.POINTER(M3Error)]),
    "m3_cuda_session_read_output_device": (ctypes.c_int, [
        ctypes.c_void_p, ctypes.c_uint32, ctypes.c_void_p, ctypes.c_size_t,
        ctypes.POINTER(M3Error)]),
    "m3_cuda_session_read_output_device_async": (ctypes.c_int, [
        ctypes.c_void_p, ctypes.c_uint32, ctypes.c_void_p, ctypes.c_size_t,
        ctypes.POINTER(M3Error)]),
    "m3_cuda_session_swap_values": (ctypes.c_int, [
        ctypes.c_void_p, ctypes.c_uint32, ctypes.c_uint32,
        ctypes.POINTER(M3Error)]),
    "m3_cuda_session_stream": (ctypes.c_void_p, [ctypes.c_void_p]),
    "m3_cuda_session_device": (ctypes.c_int, [ctypes.c_void_p]),
    "m3_cuda_session_get_plan_report": (ctypes.c_int, [
        ctypes.c_void_p, ctypes.POINTER(PlanReport), ctypes.c_char_p,
        ctypes.c_size_t, ctypes.POINTER(M3Error)]),
    "m3_cuda_graph_plan": (ctypes.c_int, [
        ctypes.c_void_p, ctypes.POINTER(CudaSessionOptions),
        ctypes.POINTER(PlanInfo), ctypes.POINTER(PlanReport), ctypes.c_char_p,
        ctypes.c_size_t, ctypes.POINTER(M3Error)]),
    "m3_cuda_backend_context_create": (ctypes.c_int, [
        ctypes.POINTER(BackendOptions), ctypes.POINTER(ctypes.c_void_p),
        ctypes.POINTER(M3Error)]),
    "m3_cuda_backend_destroy_context": (None, [ctypes.c_void_p]),
    "m3_cuda_backend_allocate": (ctypes.c_int, [
        ctypes.c_void_p, ctypes.c_size_t, ctypes.c_size_t,
        ctypes.POINTER(ctypes.c_void_p), ctypes.POINTER(ctypes.c_void_p),
        ctypes.POINTER(M3Error)]),
    "m3_cuda_backend_free_storage": (None, [ctypes.c_void_p, ctypes.c_void_p,
                                            ctypes.c_void_p]),
    "m3_cuda_backend_execute": (ctypes.c_int, [
        ctypes.c_void_p, ctypes.POINTER(Command), ctypes.c_size_t,
        ctypes.c_void_p, ctypes.POINTER(M3Error)]),
    "m3_cuda_backend_write": (ctypes.c_int, [
        ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p,
        ctypes.c_size_t, ctypes.POINTER(M3Error)]),
    "m3_cuda_backend_read": (ctypes.c_int, [
        ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p,
        ctypes.c_size_t, ctypes.POINTER(M3Error)]),
    "m3_cuda_backend_supports_kind": (ctypes.c_bool, [ctypes.c_int]),
    "m3_cuda_backend_launch_count": (ctypes.c_uint, [ctypes.c_void_p]),
    "m3_cuda_storage_is_address": (ctypes.c_void_p, [ctypes.c_void_p]),
    "m3_cuda_backend_set_stream": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p,
                                                  ctypes.POINTER(M3Error)]),
    "m3_cuda_fill_uniform_host": (ctypes.c_int, [
        ctypes.c_uint64, ctypes.c_uint64, ctypes.c_float, ctypes.c_float,
        ctypes.c_void_p, ctypes.c_size_t, ctypes.POINTER(M3Error)]),
    "m3_cuda_fill_normal_host": (ctypes.c_int, [
        ctypes.c_uint64, ctypes.c_uint64, ctypes.c_float, ctypes.c_float,
        ctypes.c_void_p, ctypes.c_size_t, ctypes.POINTER(M3Error)]),
    "m3_cuda_fill_uniform_device": (ctypes.c_int, [
        ctypes.c_uint64, ctypes.c_uint64, ctypes.c_float, ctypes.c_float,
        ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p,
        ctypes.POINTER(M3Error)]),
    "m3_cuda_fill_normal_device": (ctypes.c_int, [
        ctypes.c_uint64, ctypes.c_uint64, ctypes.c_float, ctypes.c_float,
        ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p,
        ctypes.POINTER(M3Error)]),
    "m3_cuda_device_count": (ctypes.c_int, []),
    "m3_cuda_codec_self_test": (ctypes.c_int, [
        ctypes.c_int, ctypes.POINTER(ctypes.c_uint64), ctypes.POINTER(M3Error)]),
    "m3_cuda_division_self_test": (ctypes.c_int, [
        ctypes.c_int, ctypes.c_uint64, ctypes.POINTER(ctypes.c_uint64),
        ctypes.POINTER(M3Error)]),
    "m3_cuda_sin_squared_self_test": (ctypes.c_int, [
        ctypes.c_int, ctypes.POINTER(ctypes.c_float), ctypes.POINTER(ctypes.c_uint32),
        ctypes.POINTER(M3Error)]),
    "m3_cuda_sin_squared_packed_self_test": (ctypes.c_int, [
        ctypes.c_int, ctypes.POINTER(ctypes.c_uint64), ctypes.POINTER(M3Error)]),
    "m3_cuda_exp_self_test": (ctypes.c_int, [
        ctypes.c_int, ctypes.POINTER(ctypes.c_uint32),
        ctypes.POINTER(ctypes.c_uint64), ctypes.POINTER(M3Error)]),
    "m3_cuda_shard_options_init": (None, [ctypes.POINTER(ShardOptions)]),
    "m3_cuda_shard_id_create": (ctypes.c_int, [ctypes.POINTER(ShardId),
                                               ctypes.POINTER(M3Error)]),
    "m3_cuda_shard_plan": (ctypes.c_int, [
        ctypes.c_void_p, ctypes.POINTER(ShardOptions), ctypes.c_uint32,
        ctypes.POINTER(ShardSlab), ctypes.POINTER(ctypes.c_int), ctypes.POINTER(M3Error)]),
    "m3_cuda_shard_session_create": (ctypes.c_int, [
        ctypes.POINTER(ctypes.c_void_p), ctypes.c_void_p,
        ctypes.POINTER(SessionOptions), ctypes.POINTER(CudaSessionOptions),
        ctypes.POINTER(ShardOptions), ctypes.POINTER(M3Error)]),
    "m3_cuda_shard_get_slab": (ctypes.c_int, [
        ctypes.c_void_p, ctypes.c_uint32, ctypes.POINTER(ShardSlab),
        ctypes.POINTER(M3Error)]),
    "m3_cuda_shard_write_input": (ctypes.c_int, [
        ctypes.c_void_p, ctypes.c_uint32, ctypes.c_void_p, ctypes.c_size_t,
        ctypes.c_bool, ctypes.POINTER(M3Error)]),
    "m3_cuda_shard_read_output": (ctypes.c_int, [
        ctypes.c_void_p, ctypes.c_uint32, ctypes.c_void_p, ctypes.c_size_t,
        ctypes.c_bool, ctypes.POINTER(M3Error)]),
    "m3_cuda_abs_max_static": (ctypes.c_int, [
        ctypes.c_int, ctypes.c_void_p, ctypes.c_int,
        ctypes.POINTER(ctypes.c_void_p), ctypes.POINTER(ctypes.c_uint64),
        ctypes.c_size_t, ctypes.c_void_p, ctypes.POINTER(M3Error)]),
}


def bind(lib: ctypes.CDLL, cuda: bool = True) -> ctypes.CDLL:
    """Declare argument and result types on a loaded m3.h library."""
    table = dict(_SIGNATURES)
    if cuda:
        table.update(_CUDA_SIGNATURES)
    for name, (restype, argtypes) in table.items():
        fn = getattr(lib, name)
        fn.restype = restype
        fn.argtypes = argtypes
    return lib


def load(path: str | None = None) -> ctypes.CDLL:
    """Load libm3cuda.so (once).  Raises when it has not been built."""
    global _library
    if path is None and _library is not None:
        return _library
    target = path or LIBRARY_PATH
    if not os.path.exists(target):
        raise FileNotFoundError(
            f"{target} is missing: build it with `make -C {HERE}` "
            "(the CUDA provider has no fallback)")
    lib = bind(ctypes.CDLL(target, mode=ctypes.RTLD_LOCAL), cuda=True)
    if path is None:
        _library = lib
    return lib


def check(status: int, error: M3Error) -> None:
    if status != OK:
        raise M3Failure(status, error.message.decode(errors="replace"))


class Graph:
    """m3_graph of include/m3.h:209-229."""

    def __init__(self, lib: ctypes.CDLL | None = None):
        self.lib = lib or load()
        self.handle = ctypes.c_void_p()
        self.values: list[tuple[int, tuple[int, ...], int]] = []
        err = M3Error()
        check(self.lib.m3_graph_create(ctypes.byref(self.handle),
                                       ctypes.byref(err)), err)

    def close(self) -> None:
        if self.handle:
            self.lib.m3_graph_free(self.handle)
            self.handle = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def value(self, role: int, dtype: int, shape: Sequence[int]) -> int:
        desc = GraphValueDesc()
        dims = (ctypes.c_uint64 * MAX_RANK)(*shape)
        self.lib.m3_graph_value_desc_init(ctypes.byref(desc), role, dtype,
                                          len(shape), dims)
        out = ctypes.c_uint32()
        err = M3Error()
        check(self.lib.m3_graph_add_value(self.handle, ctypes.byref(desc),
                                          ctypes.byref(out),
                                          ctypes.byref(err)), err)
        self.values.append((dtype, tuple(shape), role))
        return out.value

    def constant(self, dtype: int, array: np.ndarray) -> int:
        array = np.ascontiguousarray(array)
        vid = self.value(CONSTANT, dtype, array.shape)
        err = M3Error()
        check(self.lib.m3_graph_set_constant(
            self.handle, vid, array.ctypes.data_as(ctypes.c_void_p),
            array.nbytes, ctypes.byref(err)), err)
        return vid

    @staticmethod
    def node_desc(kind: str | int, inputs: Iterable[int],
                  outputs: Iterable[int], epsilon: float | None = None,
                  k: int | None = None) -> NodeDesc:
        desc = NodeDesc()
        desc.kind = OPS[kind] if isinstance(kind, str) else kind
        for i in range(5):
            desc.inputs[i] = VALUE_NONE
        for i in range(2):
            desc.outputs[i] = VALUE_NONE
        for i, v in enumerate(inputs):
            desc.inputs[i] = v
        for i, v in enumerate(outputs):
            desc.outputs[i] = v
        if epsilon is not None:
            desc.parameters.norm.epsilon = epsilon
        if k is not None:
            desc.parameters.top_k.k = k
        return desc

    def node(self, kind: str | int, inputs: Iterable[int],
             outputs: Iterable[int], **params) -> None:
        desc = self.node_desc(kind, inputs, outputs, **params)
        err = M3Error()
        check(self.lib.m3_graph_add_node(self.handle, ctypes.byref(desc),
                                         ctypes.byref(err)), err)

    def _shape_of(self, kind: int, inputs: list[int], k: int | None):
        """Python-side copy of the inferred shape, for read-buffer sizing."""
        first = self.values[inputs[0]][1]
        if kind in (OPS["ADD"], OPS["MUL"]):
            return tuple(np.broadcast_shapes(first, self.values[inputs[1]][1]))
        if kind == OPS["TOP_K"]:
            return first[:-1] + (k,)
        if kind == OPS["ABS_MAX"]:
            return (1,)
        if kind == OPS["ROW_SUM"]:
            return first[:-1] + (1,)
        if kind == OPS["CATEGORICAL"]:
            return first[:-1]
        return first

    def inferred(self, kind: str | int, inputs: Iterable[int], role: int,
                 dtype: int, output_index: int = 0, **params) -> int:
        inputs = list(inputs)
        desc = self.node_desc(kind, inputs, [], **params)
        out = ctypes.c_uint32(VALUE_NONE)
        err = M3Error()
        check(self.lib.m3_graph_add_inferred_value(
            self.handle, ctypes.byref(desc), output_index, role, dtype,
            ctypes.byref(out), ctypes.byref(err)), err)
        code = desc.kind
        if code in (OPS["SNAKE1D"], OPS["TANH"], OPS["CLAMP_UNIT"],
                    OPS["ABS_MAX"], OPS["ROW_SUM"]):
            dtype = F32
        elif code == OPS["COPY"]:
            dtype = self.values[inputs[0]][0]
        elif code == OPS["TOP_K"]:
            dtype = F32 if output_index == 0 else I32
        elif code == OPS["CATEGORICAL"]:
            dtype = I32
        self.values.append((dtype, self._shape_of(code, inputs,
                                                  params.get("k")), role))
        return out.value


class Session:
    """m3_session of include/m3.h:240-259 (plus the CUDA extensions when the
    library is libm3cuda.so)."""

    def __init__(self, graph: Graph, allow_metal: bool = True,
                 allow_cpu: bool = True, allow_neural_engine: bool = True,
                 device: int = -1, stream: int | None = None,
                 fuse: bool = True, cuda: bool = True, cuda_graphs: bool = True,
                 shard: ShardOptions | None = None):
        self.lib = graph.lib
        self.values = list(graph.values)
        self.handle = ctypes.c_void_p()
        self.cuda = cuda
        self.shard = shard
        options = SessionOptions(allow_neural_engine, allow_metal, allow_cpu)
        err = M3Error()
        if shard is not None:
            extra = CudaSessionOptions()
            self.lib.m3_cuda_session_options_init(ctypes.byref(extra))
            extra.device = device
            extra.stream = stream
            extra.fuse = fuse
            extra.cuda_graphs = cuda_graphs
            status = self.lib.m3_cuda_shard_session_create(
                ctypes.byref(self.handle), graph.handle, ctypes.byref(options),
                ctypes.byref(extra), ctypes.byref(shard), ctypes.byref(err))
            check(status, err)
            # reads and writes move this rank's slab: local shapes
            for vid in range(len(self.values)):
                slab = self.shard_slab(vid)
                dtype, _, role = self.values[vid]
                local = tuple(slab.local.shape[a] for a in range(slab.local.rank))
                self.values[vid] = (dtype, local, role)
            return
        if cuda:
            extra = CudaSessionOptions()
            self.lib.m3_cuda_session_options_init(ctypes.byref(extra))
            extra.device = device
            extra.stream = stream
            extra.fuse = fuse
            extra.cuda_graphs = cuda_graphs
            status = self.lib.m3_cuda_session_create(
                ctypes.byref(self.handle), graph.handle, ctypes.byref(options),
                ctypes.byref(extra), ctypes.byref(err))
        else:
            status = self.lib.m3_session_create(
                ctypes.byref(self.handle), graph.handle, ctypes.byref(options),
                ctypes.byref(err))
        check(status, err)

    def close(self) -> None:
        if self.handle:
            self.lib.m3_session_free(self.handle)
            self.handle = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def write(self, vid: int, array: np.ndarray) -> None:
        array = np.ascontiguousarray(array)
        err = M3Error()
        check(self.lib.m3_session_write_input(
            self.handle, vid, array.ctypes.data_as(ctypes.c_void_p),
            array.nbytes, ctypes.byref(err)), err)

    def read(self, vid: int, out: np.ndarray | None = None) -> np.ndarray:
        dtype, shape, _ = self.values[vid]
        if out is None:
            out = np.empty(shape, dtype=NUMPY_OF[dtype])
        err = M3Error()
        check(self.lib.m3_session_read_output(
            self.handle, vid, out.ctypes.data_as(ctypes.c_void_p), out.nbytes,
            ctypes.byref(err)), err)
        return out

    def run(self) -> None:
        err = M3Error()
        check(self.lib.m3_session_run(self.handle, ctypes.byref(err)), err)

    def run_status(self) -> tuple[int, str]:
        err = M3Error()
        status = self.lib.m3_session_run(self.handle, ctypes.byref(err))
        return status, err.message.decode(errors="replace")

    def run_async(self) -> None:
        err = M3Error()
        check(self.lib.m3_cuda_session_run_async(self.handle,
                                                 ctypes.byref(err)), err)

    def run_steps(self, count: int, carried_in: int | None = None,
                  carried_out: int | None = None) -> None:
        """m3_cuda_session_run_steps_async: `count` runs, exchanging
        carried_in and carried_out between consecutive runs."""
        none = 0xFFFFFFFF
        err = M3Error()
        check(self.lib.m3_cuda_session_run_steps_async(
            self.handle, count, none if carried_in is None else carried_in,
            none if carried_out is None else carried_out, ctypes.byref(err)), err)

    def submit_host(self, inputs: dict, outputs: dict) -> None:
        """m3_cuda_session_submit_host_async: {value id: host pointer} for
        inputs and outputs (pinned memory for asynchronous copies); the
        buffers must stay valid until synchronize()."""
        ni, no = len(inputs), len(outputs)
        in_ids = (ctypes.c_uint32 * max(ni, 1))(*inputs.keys())
        in_ptr = (ctypes.c_void_p * max(ni, 1))(*inputs.values())
        out_ids = (ctypes.c_uint32 * max(no, 1))(*outputs.keys())
        out_ptr = (ctypes.c_void_p * max(no, 1))(*outputs.values())
        err = M3Error()
        check(self.lib.m3_cuda_session_submit_host_async(
            self.handle, ni, in_ids, in_ptr, no, out_ids, out_ptr, ctypes.byref(err)), err)

    def synchronize(self) -> None:
        err = M3Error()
        check(self.lib.m3_cuda_session_synchronize(self.handle,
                                                   ctypes.byref(err)), err)

    def plan_info(self) -> PlanInfo:
        info = PlanInfo()
        err = M3Error()
        check(self.lib.m3_session_get_plan_info(
            self.handle, ctypes.byref(info), ctypes.byref(err)), err)
        return info

    def provider(self, node: int) -> int:
        out = ctypes.c_int(-1)
        err = M3Error()
        check(self.lib.m3_session_get_node_provider(
            self.handle, node, ctypes.byref(out), ctypes.byref(err)), err)
        return out.value

    def plan_report(self) -> tuple[PlanReport, str]:
        report = PlanReport()
        text = ctypes.create_string_buffer(4096)
        err = M3Error()
        check(self.lib.m3_cuda_session_get_plan_report(
            self.handle, ctypes.byref(report), text, len(text),
            ctypes.byref(err)), err)
        return report, text.value.decode()

    def device_pointer(self, vid: int) -> int:
        ptr = ctypes.c_void_p()
        size = ctypes.c_size_t()
        err = M3Error()
        check(self.lib.m3_cuda_session_value_device_pointer(
            self.handle, vid, ctypes.byref(ptr), ctypes.byref(size),
            ctypes.byref(err)), err)
        return ptr.value or 0

    def write_device(self, vid: int, pointer: int, nbytes: int) -> None:
        err = M3Error()
        check(self.lib.m3_cuda_session_write_input_device(
            self.handle, vid, ctypes.c_void_p(pointer), nbytes,
            ctypes.byref(err)), err)

    def read_device(self, vid: int, pointer: int, nbytes: int) -> None:
        err = M3Error()
        check(self.lib.m3_cuda_session_read_output_device(
            self.handle, vid, ctypes.c_void_p(pointer), nbytes,
            ctypes.byref(err)), err)

    def read_device_async(self, vid: int, pointer: int, nbytes: int) -> None:
        """m3_cuda_session_read_output_device_async: stream-ordered copy of
        an output into device memory, no host wait."""
        err = M3Error()
        check(self.lib.m3_cuda_session_read_output_device_async(
            self.handle, vid, ctypes.c_void_p(pointer), nbytes, ctypes.byref(err)), err)

    def value_bytes(self, vid: int) -> int:
        """Bytes of a value on this session (a shard's local slab)."""
        dtype, shape, _ = self.values[vid]
        return int(np.prod(shape, dtype=np.int64)) * ITEMSIZE[dtype]

    def shard_slab(self, vid: int) -> ShardSlab:
        slab = ShardSlab()
        err = M3Error()
        check(self.lib.m3_cuda_shard_get_slab(self.handle, vid, ctypes.byref(slab),
                                              ctypes.byref(err)), err)
        return slab

    def shard_write(self, vid: int, pointer: int, global_bytes: int,
                    device: bool = False) -> None:
        """This rank's slab of an input out of a buffer laid out as the
        global tensor (host or device memory)."""
        err = M3Error()
        check(self.lib.m3_cuda_shard_write_input(
            self.handle, vid, ctypes.c_void_p(pointer), global_bytes, device,
            ctypes.byref(err)), err)

    def shard_read(self, vid: int, pointer: int, global_bytes: int,
                   device: bool = False) -> None:
        """This rank's slab of an output into its place in a global buffer."""
        err = M3Error()
        check(self.lib.m3_cuda_shard_read_output(
            self.handle, vid, ctypes.c_void_p(pointer), global_bytes, device,
            ctypes.byref(err)), err)

    def swap(self, input_vid: int, output_vid: int) -> None:
        err = M3Error()
        check(self.lib.m3_cuda_session_swap_values(
            self.handle, input_vid, output_vid, ctypes.byref(err)), err)

    @property
    def stream(self) -> int:
        return self.lib.m3_cuda_session_stream(self.handle) or 0


def graph_plan(graph: Graph, fuse: bool = True):
    """Host-only compile of a graph: (PlanInfo, PlanReport, description)."""
    lib = graph.lib
    options = CudaSessionOptions()
    lib.m3_cuda_session_options_init(ctypes.byref(options))
    options.fuse = fuse
    info = PlanInfo()
    report = PlanReport()
    text = ctypes.create_string_buffer(4096)
    err = M3Error()
    check(lib.m3_cuda_graph_plan(graph.handle, ctypes.byref(options),
                                 ctypes.byref(info), ctypes.byref(report),
                                 text, len(text), ctypes.byref(err)), err)
    return info, report, text.value.decode()


def fill_uniform(seed: int, sequence: int, low: float, high: float,
                 count: int) -> np.ndarray:
    """The reference RNG's uniform stream scaled to [low, high) (host)."""
    out = np.empty(count, dtype=np.float32)
    err = M3Error()
    check(load().m3_cuda_fill_uniform_host(
        seed, sequence, low, high, out.ctypes.data_as(ctypes.c_void_p), count,
        ctypes.byref(err)), err)
    return out


def fill_normal(seed: int, sequence: int, mean: float, deviation: float,
                count: int) -> np.ndarray:
    """The reference RNG's Box-Muller normals, mean + deviation * z (host)."""
    out = np.empty(count, dtype=np.float32)
    err = M3Error()
    check(load().m3_cuda_fill_normal_host(
        seed, sequence, mean, deviation, out.ctypes.data_as(ctypes.c_void_p),
        count, ctypes.byref(err)), err)
    return out


def shard_id() -> ShardId:
    """m3_cuda_shard_id_create: a new communicator id (rank 0)."""
    out = ShardId()
    err = M3Error()
    check(load().m3_cuda_shard_id_create(ctypes.byref(out), ctypes.byref(err)), err)
    return out


def shard_plan(graph: Graph, rank: int, count: int, axis: int, vid: int):
    """m3_cuda_shard_plan (host only): (slab, chosen axis) of one value."""
    options = ShardOptions(rank, count, axis, None)
    slab = ShardSlab()
    chosen = ctypes.c_int(-1)
    err = M3Error()
    check(graph.lib.m3_cuda_shard_plan(graph.handle, ctypes.byref(options), vid,
                                       ctypes.byref(slab), ctypes.byref(chosen),
                                       ctypes.byref(err)), err)
    return slab, chosen.value


ABS_MAX_STATIC_MAX_TENSORS = 64


def abs_max_static(dtype: int, pointers, counts, maxima: int, device: int = 0,
                   stream: int = 0) -> None:
    """m3_cuda_abs_max_static: max |x| of each device tensor into `maxima`
    (a device F32 array), using no allocation; see include/m3_cuda.h.
    Raises M3Failure with the library's status and message."""
    n = len(pointers)
    if len(counts) != n:
        raise ValueError("one element count per input pointer")
    inputs = (ctypes.c_void_p * max(n, 1))(*pointers)
    sizes = (ctypes.c_uint64 * max(n, 1))(*counts)
    err = M3Error()
    check(load().m3_cuda_abs_max_static(device, stream, dtype, inputs, sizes,
                                        n, maxima, ctypes.byref(err)), err)
