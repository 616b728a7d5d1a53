"""ctypes binding of libdiskllm_cuda.so (include/diskllm_cuda.h, include/sampler.h).

This is the Python host side above the C ABI.  It mirrors DiskLLM's sampler interface
(include/sampler.h:7-34: sampler_create / sampler_free / sampler_apply_*_penalty /
sampler_sample / greedy_sample) and adds the batched device entry point.  The library is
required: loading it on a machine without the built .so raises, and nothing here falls back
to a host implementation.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libdiskllm_cuda.so")

DLLM_OK = 0
DLLM_ERR_INVALID_ARG = 1
DLLM_ERR_OOM = 2
DLLM_ERR_UNSUPPORTED = 6
STATUS_NAMES = {0: "OK", 1: "INVALID_ARG", 2: "OOM", 3: "CUDA", 4: "NCCL", 5: "TIMEOUT",
                6: "UNSUPPORTED"}
DTYPE_F32 = 0
DTYPE_BF16 = 1
MODE_TOPP_SORTED = 0x1
MODE_PEN_TRUE_DIV = 0x2
MODE_MINP_RELATIVE = 0x4
ROW_ERR_HIST_TABLE = 1
ROW_ERR_NONFINITE = 2
ROW_ERR_TOPK_LARGE = 4
ROW_ERR_WALK = 8
ROW_ERR_TIMEOUT = 16
ROW_TOPP_EDGE = 32  # information: the index-order top-p cut lies near the threshold

# every symbol the public headers declare
EXPORTS = [
    "dllm_cuda_sample_batch", "dllm_cuda_version", "dllm_cuda_last_error",
    "dllm_cuda_set_debug_counters", "dllm_cuda_workspace_bytes", "dllm_cuda_sample_batch_static",
    "dllm_cuda_set_timing_events", "dllm_cuda_shard_candidates", "dllm_cuda_merge_sample",
    "dllm_cuda_append_history", "dllm_cuda_lmhead_logits",
    "dllm_cuda_debug_inject_wait_timeout", "dllm_cuda_debug_fail_allocations",
    "dllm_cuda_peer_exchange_create", "dllm_cuda_peer_exchange_open", "dllm_cuda_peer_exchange_close",
    "dllm_cuda_peer_exchange_free", "dllm_cuda_shard_candidates_peer", "dllm_cuda_merge_sample_peer",
    "diskllm_grammar_init_from_file", "diskllm_grammar_init_from_str", "diskllm_grammar_init_json",
    "diskllm_grammar_free", "diskllm_grammar_reset", "diskllm_grammar_accept_str", "diskllm_grammar_advance",
    "diskllm_grammar_is_finished", "diskllm_grammar_apply_mask", "dllm_grammar_build_bitmask",
    "dllm_grammar_vocab_create", "dllm_grammar_vocab_free", "dllm_grammar_build_bitmask_cached",
    "dllm_sampler_get_rng_state", "dllm_sampler_set_rng_state",
    "sampler_create", "sampler_free", "sampler_apply_repetition_penalty",
    "sampler_apply_presence_penalty", "sampler_sample", "greedy_sample",
]


class DllmError(RuntimeError):
    pass


class SamplerParams(C.Structure):
    """dllm_sampler_params"""
    _fields_ = [
        ("temperature", C.c_float),
        ("top_p", C.c_float),
        ("min_p", C.c_float),
        ("top_k", C.c_int),
        ("repetition", C.c_float),
        ("presence", C.c_float),
        ("frequency", C.c_float),
    ]


class SamplerConfig(C.Structure):
    """sampler_config (DiskLLM include/sampler.h:10-16)"""
    _fields_ = [
        ("temperature", C.c_float),
        ("top_k", C.c_int),
        ("top_p", C.c_float),
        ("min_p", C.c_float),
        ("seed", C.c_uint64),
    ]


class BatchDesc(C.Structure):
    """dllm_batch_desc"""
    _fields_ = [
        ("rows", C.c_int),
        ("vocab", C.c_int),
        ("row_stride", C.c_int64),
        ("dtype", C.c_int),
        ("logits", C.c_void_p),
        ("mask", C.c_void_p),
        ("mask_stride", C.c_int64),
        ("hist_ids", C.c_void_p),
        ("hist_off", C.c_void_p),
        ("hist_max", C.c_int),
        ("uniforms", C.c_void_p),
        ("params", SamplerParams),
        ("row_params", C.c_void_p),
        ("topk_max", C.c_int),
        ("flags", C.c_uint),
        ("token", C.c_void_p),
        ("probs", C.c_void_p),
        ("probs_stride", C.c_int64),
        ("pen_logits", C.c_void_p),
        ("pen_stride", C.c_int64),
        ("status", C.c_void_p),
        ("topk_ids", C.c_void_p),
        ("topk_stride", C.c_int64),
        ("workspace", C.c_void_p),
        ("workspace_bytes", C.c_size_t),
    ]


_lib = None


def load_library(path: str = LIB_PATH) -> C.CDLL:
    """Loads libdiskllm_cuda.so; raises if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        raise DllmError(f"{path} is missing: build it with `python -m diskllm_b200.build`")
    lib = C.CDLL(path)
    lib.dllm_cuda_sample_batch.restype = C.c_int
    lib.dllm_cuda_sample_batch.argtypes = [C.POINTER(BatchDesc), C.c_void_p]
    lib.dllm_cuda_set_debug_counters.restype = C.c_int
    lib.dllm_cuda_set_debug_counters.argtypes = [C.c_void_p]
    lib.dllm_cuda_shard_candidates.restype = C.c_int
    lib.dllm_cuda_shard_candidates.argtypes = [C.POINTER(BatchDesc), C.c_int64, C.c_int64, C.c_int,
                                               C.c_void_p, C.c_void_p, C.c_void_p]
    lib.dllm_cuda_merge_sample.restype = C.c_int
    lib.dllm_cuda_merge_sample.argtypes = [C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_void_p,
                                           C.POINTER(SamplerParams), C.c_void_p, C.c_void_p, C.c_void_p,
                                           C.c_void_p, C.c_void_p]
    lib.dllm_cuda_lmhead_logits.restype = C.c_int
    lib.dllm_cuda_lmhead_logits.argtypes = [C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_float, C.c_int,
                                            C.c_void_p, C.c_int, C.c_float, C.c_void_p, C.c_void_p]
    lib.dllm_cuda_append_history.restype = C.c_int
    lib.dllm_cuda_append_history.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int64, C.c_void_p]
    lib.dllm_cuda_set_timing_events.restype = C.c_int
    lib.dllm_cuda_set_timing_events.argtypes = [C.c_void_p, C.c_void_p]
    lib.dllm_cuda_sample_batch_static.restype = C.c_int
    lib.dllm_cuda_sample_batch_static.argtypes = [C.POINTER(BatchDesc), C.c_void_p]
    lib.dllm_cuda_debug_inject_wait_timeout.restype = C.c_int
    lib.dllm_cuda_debug_inject_wait_timeout.argtypes = [C.c_int, C.c_longlong]
    lib.dllm_cuda_debug_fail_allocations.restype = C.c_int
    lib.dllm_cuda_debug_fail_allocations.argtypes = [C.c_int]
    for name, args in (("dllm_cuda_peer_exchange_create", [C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_void_p]),
                       ("dllm_cuda_peer_exchange_open", [C.c_void_p, C.c_void_p]),
                       ("dllm_cuda_peer_exchange_close", [C.c_void_p]),
                       ("dllm_cuda_peer_exchange_free", [C.c_void_p]),
                       ("dllm_cuda_shard_candidates_peer", [C.POINTER(BatchDesc), C.c_int64, C.c_int64, C.c_int,
                                                            C.c_void_p, C.c_int, C.c_int, C.c_uint64, C.c_void_p]),
                       ("dllm_cuda_merge_sample_peer", [C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_uint64,
                                                        C.POINTER(SamplerParams), C.c_void_p, C.c_void_p, C.c_void_p,
                                                        C.c_void_p, C.c_void_p])):
        f = getattr(lib, name)
        f.restype = C.c_int
        f.argtypes = args
    lib.dllm_cuda_workspace_bytes.restype = C.c_size_t
    lib.dllm_cuda_workspace_bytes.argtypes = [C.POINTER(BatchDesc)]
    lib.dllm_cuda_version.restype = C.c_char_p
    lib.dllm_cuda_last_error.restype = C.c_char_p
    lib.dllm_sampler_get_rng_state.restype = C.c_uint64
    lib.dllm_sampler_get_rng_state.argtypes = [C.c_void_p]
    lib.dllm_sampler_set_rng_state.restype = None
    lib.dllm_sampler_set_rng_state.argtypes = [C.c_void_p, C.c_uint64]
    lib.sampler_create.restype = C.c_void_p
    lib.sampler_create.argtypes = [C.POINTER(SamplerConfig)]
    lib.sampler_free.restype = None
    lib.sampler_free.argtypes = [C.c_void_p]
    lib.sampler_sample.restype = C.c_int
    lib.sampler_sample.argtypes = [C.c_void_p, C.c_void_p, C.c_int]
    lib.greedy_sample.restype = C.c_int
    lib.greedy_sample.argtypes = [C.c_void_p, C.c_int]
    for name in ("sampler_apply_repetition_penalty", "sampler_apply_presence_penalty"):
        f = getattr(lib, name)
        f.restype = None
        f.argtypes = [C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_float]
    _lib = lib
    return lib


def set_timing_events(before=None, after=None):
    """Has every later sampling call record the two torch.cuda.Event objects right before and
    right after the cluster kernel (None, None switches it off)."""
    b = None if before is None else before.cuda_event
    a = None if after is None else after.cuda_event
    rc = load_library().dllm_cuda_set_timing_events(b, a)
    if rc != DLLM_OK:
        raise DllmError(f"dllm_cuda_set_timing_events: {STATUS_NAMES.get(rc, rc)}")


FAULT_NONE, FAULT_COPY_WAIT, FAULT_EXCHANGE_WAIT = 0, 1, 2


def inject_wait_timeout(site: int, polls: int = 1) -> None:
    """Test hook: later sampling launches make one bounded wait run out (FAULT_COPY_WAIT or
    FAULT_EXCHANGE_WAIT) after `polls` polls; FAULT_NONE switches it off."""
    rc = load_library().dllm_cuda_debug_inject_wait_timeout(int(site), int(polls))
    if rc != DLLM_OK:
        raise DllmError(f"dllm_cuda_debug_inject_wait_timeout: {STATUS_NAMES.get(rc, rc)}")


def fail_allocations(count: int) -> None:
    """Test hook: the library's next `count` device allocations fail as out of memory."""
    rc = load_library().dllm_cuda_debug_fail_allocations(int(count))
    if rc != DLLM_OK:
        raise DllmError(f"dllm_cuda_debug_fail_allocations: {STATUS_NAMES.get(rc, rc)}")


def set_debug_counters(tensor_or_none):
    """Points the kernels' diagnostic counters at a zeroed CUDA int64 tensor of >= 32 entries
    (or switches them off with None)."""
    ptr = None if tensor_or_none is None else tensor_or_none.data_ptr()
    rc = load_library().dllm_cuda_set_debug_counters(ptr)
    if rc != DLLM_OK:
        raise DllmError(f"dllm_cuda_set_debug_counters: {STATUS_NAMES.get(rc, rc)}")


def version() -> str:
    return load_library().dllm_cuda_version().decode()


def make_params(temperature=1.0, top_p=1.0, min_p=0.0, top_k=0, repetition=1.0, presence=0.0,
                frequency=0.0) -> SamplerParams:
    return SamplerParams(float(temperature), float(top_p), float(min_p), int(top_k),
                         float(repetition), float(presence), float(frequency))


# ---------------------------------------------------------------------------------------------
# drop-in sampler (host pointers, like DiskLLM's sampler.h)

class Sampler:
    """DiskLLM's `sampler` object (src/sampler.c:56-95) served by the CUDA library."""

    def __init__(self, temperature=0.7, top_k=40, top_p=0.9, min_p=0.0, seed=0):
        self._lib = load_library()
        cfg = SamplerConfig(float(temperature), int(top_k), float(top_p), float(min_p), int(seed))
        self._h = self._lib.sampler_create(C.byref(cfg))
        if not self._h:
            raise DllmError("sampler_create returned NULL")

    def close(self):
        if self._h:
            self._lib.sampler_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def rng_state(self) -> int:
        return int(self._lib.dllm_sampler_get_rng_state(self._h))

    @rng_state.setter
    def rng_state(self, v: int):
        self._lib.dllm_sampler_set_rng_state(self._h, int(v))

    def sample(self, logits: np.ndarray) -> int:
        a = np.ascontiguousarray(logits, dtype=np.float32)
        return int(self._lib.sampler_sample(self._h, a.ctypes.data, a.shape[0]))


def greedy_sample(logits: np.ndarray) -> int:
    a = np.ascontiguousarray(logits, dtype=np.float32)
    return int(load_library().greedy_sample(a.ctypes.data, a.shape[0]))


def apply_repetition_penalty(logits: np.ndarray, seen, penalty: float) -> None:
    """In place on a float32 numpy row, like src/sampler.c:21-33."""
    assert logits.dtype == np.float32 and logits.flags.c_contiguous
    ids = np.ascontiguousarray(seen, dtype=np.int32)
    load_library().sampler_apply_repetition_penalty(logits.ctypes.data, logits.shape[0],
                                                    ids.ctypes.data, ids.shape[0], penalty)


def apply_presence_penalty(logits: np.ndarray, seen, presence: float) -> None:
    """In place on a float32 numpy row, like src/sampler.c:35-52."""
    assert logits.dtype == np.float32 and logits.flags.c_contiguous
    ids = np.ascontiguousarray(seen, dtype=np.int32)
    load_library().sampler_apply_presence_penalty(logits.ctypes.data, logits.shape[0],
                                                  ids.ctypes.data, ids.shape[0], presence)


# ---------------------------------------------------------------------------------------------
# batched device entry point (torch tensors are only containers for device memory here)

def fill_desc(logits, uniforms, params=None, *, mask=None, hist_ids=None, hist_off=None,
              hist_max=None, row_params=None, topk_max=0, flags=0, token=None, probs=None,
              pen_logits=None, status=None, topk_ids=None, workspace=None) -> tuple[BatchDesc, object]:
    """Builds a dllm_batch_desc from CUDA tensors; returns (desc, token tensor)."""
    import torch

    assert logits.is_cuda and logits.dim() == 2
    rows, vocab = logits.shape
    if logits.dtype == torch.float32:
        dt = DTYPE_F32
    elif logits.dtype == torch.bfloat16:
        dt = DTYPE_BF16
    else:
        raise TypeError(f"unsupported logits dtype {logits.dtype}")
    assert logits.stride(1) == 1
    if token is None:
        token = torch.empty(rows, dtype=torch.int32, device=logits.device)
    if params is None:
        params = make_params()
    elif isinstance(params, dict):
        params = make_params(**params)
    d = BatchDesc()
    d.rows, d.vocab, d.row_stride, d.dtype = rows, vocab, logits.stride(0), dt
    d.logits = logits.data_ptr()
    if mask is not None:
        assert mask.dtype in (torch.int32, torch.uint32) and mask.is_cuda
        d.mask, d.mask_stride = mask.data_ptr(), mask.stride(0)
    if hist_ids is not None:
        assert hist_ids.dtype == torch.int32 and hist_off.dtype == torch.int64
        d.hist_ids, d.hist_off = hist_ids.data_ptr(), hist_off.data_ptr()
        if hist_max is None:
            hist_max = int((hist_off[1:] - hist_off[:-1]).max().item()) if rows else 0
        d.hist_max = int(hist_max)
    assert uniforms.dtype == torch.float32 and uniforms.is_cuda
    d.uniforms = uniforms.data_ptr()
    d.params = params
    if row_params is not None:
        d.row_params = row_params.data_ptr()
        d.topk_max = int(topk_max)
    d.flags = int(flags)
    d.token = token.data_ptr()
    if probs is not None:
        d.probs, d.probs_stride = probs.data_ptr(), probs.stride(0)
    if pen_logits is not None:
        d.pen_logits, d.pen_stride = pen_logits.data_ptr(), pen_logits.stride(0)
    if status is not None:
        d.status = status.data_ptr()
    if topk_ids is not None:
        d.topk_ids, d.topk_stride = topk_ids.data_ptr(), topk_ids.stride(0)
    if workspace is not None:
        d.workspace, d.workspace_bytes = workspace.data_ptr(), workspace.numel() * workspace.element_size()
    return d, token


def workspace_bytes(logits, uniforms, params=None, **kw) -> int:
    """dllm_cuda_workspace_bytes for the same arguments as sample_batch."""
    d, _ = fill_desc(logits, uniforms, params, **kw)
    return int(load_library().dllm_cuda_workspace_bytes(C.byref(d)))


def sample_batch(logits, uniforms, params=None, *, stream=None, check=True, **kw):
    """Calls dllm_cuda_sample_batch on CUDA tensors.  Returns the int32 token tensor."""
    import torch

    d, token = fill_desc(logits, uniforms, params, **kw)
    if stream is None:
        stream = torch.cuda.current_stream(logits.device).cuda_stream
    rc = load_library().dllm_cuda_sample_batch(C.byref(d), C.c_void_p(stream))
    if check and rc != DLLM_OK:
        raise DllmError(f"dllm_cuda_sample_batch: {STATUS_NAMES.get(rc, rc)} "
                        f"({load_library().dllm_cuda_last_error().decode()})")
    return token


def sample_batch_static(logits, uniforms, params=None, *, stream=None, check=True, **kw):
    """Calls dllm_cuda_sample_batch_static: the same sampling with the library's fixed scratch
    array instead of any allocation.  Returns (token tensor, status code)."""
    import torch

    d, token = fill_desc(logits, uniforms, params, **kw)
    if stream is None:
        stream = torch.cuda.current_stream(logits.device).cuda_stream
    rc = load_library().dllm_cuda_sample_batch_static(C.byref(d), C.c_void_p(stream))
    if check and rc != DLLM_OK:
        raise DllmError(f"dllm_cuda_sample_batch_static: {STATUS_NAMES.get(rc, rc)} "
                        f"({load_library().dllm_cuda_last_error().decode()})")
    return token, rc


def params_array(rows_params, device):
    """list of dicts -> device tensor laid out as dllm_sampler_params[rows]"""
    import torch

    arr = (SamplerParams * len(rows_params))(*[make_params(**p) for p in rows_params])
    raw = np.frombuffer(bytes(arr), dtype=np.uint8).copy()
    return torch.from_numpy(raw).to(device)


def shard_candidates(logits, vocab_offset, vocab_total, k, params=None, *, stream=None, check=True, out=None,
                     **kw):
    """Step 1 of vocabulary-sharded sampling on this GPU's columns: returns (values float32
    [rows][k], global ids int32 [rows][k]) of each row's k best entries after mask and penalties.
    `logits` holds columns [vocab_offset, vocab_offset + logits.shape[1]); `mask` (if given) the
    words of those columns; history ids are global.  `out` = (vals, ids): contiguous [rows][k]
    tensors to write into (views of one buffer, for a single all-gather)."""
    import torch

    rows = logits.shape[0]
    dummy_u = torch.empty(max(rows, 1), dtype=torch.float32, device=logits.device)
    d, _ = fill_desc(logits, dummy_u, params, **kw)
    if out is not None:
        vals, ids = out
        assert vals.is_contiguous() and ids.is_contiguous() and vals.shape == (rows, k) and ids.shape == (rows, k)
        assert vals.dtype == torch.float32 and ids.dtype == torch.int32
    else:
        vals = torch.empty(rows, k, dtype=torch.float32, device=logits.device)
        ids = torch.empty(rows, k, dtype=torch.int32, device=logits.device)
    s = stream if stream is not None else torch.cuda.current_stream(logits.device).cuda_stream
    rc = load_library().dllm_cuda_shard_candidates(C.byref(d), int(vocab_offset), int(vocab_total), int(k),
                                                   vals.data_ptr(), ids.data_ptr(), s)
    if check and rc != DLLM_OK:
        raise DllmError(f"dllm_cuda_shard_candidates: {STATUS_NAMES.get(rc, rc)} ({load_library().dllm_cuda_last_error().decode()})")
    return vals, ids


def _check(rc, name):
    if rc != DLLM_OK:
        raise DllmError(f"{name}: {STATUS_NAMES.get(rc, rc)} ({load_library().dllm_cuda_last_error().decode()})")


def peer_exchange_create(rows, k, world):
    """This rank's peer exchange buffer: (device pointer, 64-byte IPC handle as bytes)."""
    buf = C.c_void_p()
    h = (C.c_ubyte * 64)()
    _check(load_library().dllm_cuda_peer_exchange_create(int(rows), int(k), int(world), C.byref(buf), h),
           "dllm_cuda_peer_exchange_create")
    return buf.value, bytes(h)


def peer_exchange_open(handle: bytes):
    """Maps another rank's exchange buffer on this GPU; returns its device pointer here."""
    h = (C.c_ubyte * 64).from_buffer_copy(handle)
    p = C.c_void_p()
    _check(load_library().dllm_cuda_peer_exchange_open(h, C.byref(p)), "dllm_cuda_peer_exchange_open")
    return p.value


def shard_candidates_peer(logits, vocab_offset, vocab_total, k, params, peers_dev, rank, world, epoch, *,
                          stream=None, **kw):
    """dllm_cuda_shard_candidates_peer: this GPU's candidates of step `epoch` into every rank's
    exchange buffer (peers_dev: int64 CUDA tensor [world] of the buffers as mapped here)."""
    import torch

    rows = logits.shape[0]
    dummy_u = torch.empty(max(rows, 1), dtype=torch.float32, device=logits.device)
    d, _ = fill_desc(logits, dummy_u, params, **kw)
    s = stream if stream is not None else torch.cuda.current_stream(logits.device).cuda_stream
    _check(load_library().dllm_cuda_shard_candidates_peer(C.byref(d), int(vocab_offset), int(vocab_total), int(k),
                                                          peers_dev.data_ptr(), int(rank), int(world), int(epoch), s),
           "dllm_cuda_shard_candidates_peer")


def shard_candidates_peer_desc(desc, vocab_offset, vocab_total, k, peers_dev, rank, world, epoch, stream):
    """dllm_cuda_shard_candidates_peer on a batch descriptor already built by fill_desc (its
    uniforms and token fields are not read); `stream` is a raw cudaStream_t value."""
    _check(load_library().dllm_cuda_shard_candidates_peer(C.byref(desc), int(vocab_offset), int(vocab_total), int(k),
                                                          peers_dev.data_ptr(), int(rank), int(world), int(epoch),
                                                          stream),
           "dllm_cuda_shard_candidates_peer")


def merge_sample_peer(rows, world, k, local_buf, epoch, uniforms, params, *, row_params=None, token=None,
                      status=None, stream=None):
    """dllm_cuda_merge_sample_peer over this rank's exchange buffer for step `epoch`."""
    import torch

    if isinstance(params, dict):
        params = make_params(**params)
    if token is None:
        token = torch.empty(rows, dtype=torch.int32, device=uniforms.device)
    s = stream if stream is not None else torch.cuda.current_stream(uniforms.device).cuda_stream
    rp = row_params.data_ptr() if row_params is not None else None
    st = status.data_ptr() if status is not None else None
    _check(load_library().dllm_cuda_merge_sample_peer(int(rows), int(world), int(k), local_buf, int(epoch),
                                                      C.byref(params), rp, uniforms.data_ptr(), token.data_ptr(), st, s),
           "dllm_cuda_merge_sample_peer")
    return token


def merge_sample(vals, ids, uniforms, params=None, *, row_params=None, token=None, status=None, stream=None,
                 check=True):
    """Step 3: tokens from all-gathered candidates vals / ids [nshards][rows][k].  `status` (int32
    [rows], optional) receives DLLM_ROW_ERR_TOPK_LARGE for per-row params the candidates cannot
    serve (temperature > 0 with top_k outside 1..k); those rows get the greedy token."""
    import torch

    nsh, rows, k = vals.shape
    assert vals.dtype == torch.float32 and ids.dtype == torch.int32 and vals.is_contiguous() and ids.is_contiguous()
    if params is None:
        params = make_params()
    elif isinstance(params, dict):
        params = make_params(**params)
    if token is None:
        token = torch.empty(rows, dtype=torch.int32, device=vals.device)
    s = stream if stream is not None else torch.cuda.current_stream(vals.device).cuda_stream
    rp = row_params.data_ptr() if row_params is not None else None
    st = status.data_ptr() if status is not None else None
    rc = load_library().dllm_cuda_merge_sample(rows, nsh, k, vals.data_ptr(), ids.data_ptr(), C.byref(params), rp,
                                               uniforms.data_ptr(), token.data_ptr(), st, s)
    if check and rc != DLLM_OK:
        raise DllmError(f"dllm_cuda_merge_sample: {STATUS_NAMES.get(rc, rc)} ({load_library().dllm_cuda_last_error().decode()})")
    return token


# ---- grammar constraint (include/grammar.h) -------------------------------------------------

TOKEN_STR_CB = C.CFUNCTYPE(C.c_void_p, C.c_void_p, C.c_int)  # returns const char *


def _grammar_lib():
    lib = load_library()
    if not getattr(lib, "_grammar_typed", False):
        lib.diskllm_grammar_init_from_str.restype = C.c_void_p
        lib.diskllm_grammar_init_from_str.argtypes = [C.c_char_p]
        lib.diskllm_grammar_init_from_file.restype = C.c_void_p
        lib.diskllm_grammar_init_from_file.argtypes = [C.c_char_p]
        lib.diskllm_grammar_init_json.restype = C.c_void_p
        lib.diskllm_grammar_init_json.argtypes = []
        lib.diskllm_grammar_free.argtypes = [C.c_void_p]
        lib.diskllm_grammar_reset.argtypes = [C.c_void_p]
        lib.diskllm_grammar_accept_str.restype = C.c_bool
        lib.diskllm_grammar_accept_str.argtypes = [C.c_void_p, C.c_char_p]
        lib.diskllm_grammar_advance.argtypes = [C.c_void_p, C.c_char_p]
        lib.diskllm_grammar_is_finished.restype = C.c_bool
        lib.diskllm_grammar_is_finished.argtypes = [C.c_void_p]
        lib.diskllm_grammar_apply_mask.restype = C.c_int
        lib.diskllm_grammar_apply_mask.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, TOKEN_STR_CB, C.c_int]
        lib.dllm_grammar_build_bitmask.restype = C.c_int
        lib.dllm_grammar_build_bitmask.argtypes = [C.c_void_p, C.c_int, C.c_void_p, TOKEN_STR_CB, C.c_int, C.c_void_p]
        lib.dllm_grammar_vocab_create.restype = C.c_void_p
        lib.dllm_grammar_vocab_create.argtypes = [C.c_int, C.c_void_p, TOKEN_STR_CB, C.c_int]
        lib.dllm_grammar_vocab_free.argtypes = [C.c_void_p]
        lib.dllm_grammar_build_bitmask_cached.restype = C.c_int
        lib.dllm_grammar_build_bitmask_cached.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p]
        lib._grammar_typed = True
    return lib


class Grammar:
    """DiskLLM's grammar constraint (diskllm_grammar_*) with the bitmask builder."""

    def __init__(self, text: str | None = None, *, json_mode: bool = False):
        lib = _grammar_lib()
        self._lib = lib
        self._g = lib.diskllm_grammar_init_json() if json_mode else lib.diskllm_grammar_init_from_str(
            text.encode() if text is not None else None)
        if not self._g:
            raise DllmError("diskllm_grammar_init failed")

    def __del__(self):
        if getattr(self, "_g", None):
            self._lib.diskllm_grammar_free(self._g)
            self._g = None

    def reset(self):
        self._lib.diskllm_grammar_reset(self._g)

    def accept(self, piece: bytes) -> bool:
        return bool(self._lib.diskllm_grammar_accept_str(self._g, piece))

    def advance(self, piece: bytes):
        self._lib.diskllm_grammar_advance(self._g, piece)

    def finished(self) -> bool:
        return bool(self._lib.diskllm_grammar_is_finished(self._g))

    def bitmask(self, pieces, eos: int) -> tuple[np.ndarray, int]:
        """(uint32 words, allowed count) for a vocabulary given as a list of bytes (None: no piece)."""
        cb, keep = _pieces_callback(pieces)
        words = np.zeros((len(pieces) + 31) // 32, dtype=np.uint32)
        n = self._lib.dllm_grammar_build_bitmask(self._g, len(pieces), None, cb, eos, words.ctypes.data)
        return words, n

    def apply_mask(self, logits: np.ndarray, pieces, eos: int) -> int:
        cb, keep = _pieces_callback(pieces)
        assert logits.dtype == np.float32 and logits.flags.c_contiguous
        return self._lib.diskllm_grammar_apply_mask(self._g, logits.ctypes.data, len(pieces), None, cb, eos)


class GrammarVocab:
    """Pieces read once (dllm_grammar_vocab_create) for per-step bitmasks without callbacks."""

    def __init__(self, pieces, eos: int):
        lib = _grammar_lib()
        self._lib = lib
        cb, keep = _pieces_callback(pieces)
        self.n = len(pieces)
        self._v = lib.dllm_grammar_vocab_create(len(pieces), None, cb, eos)
        if not self._v:
            raise DllmError("dllm_grammar_vocab_create failed")

    def __del__(self):
        if getattr(self, "_v", None):
            self._lib.dllm_grammar_vocab_free(self._v)
            self._v = None

    def bitmask(self, grammar: Grammar, out: np.ndarray | None = None) -> tuple[np.ndarray, int]:
        words = out if out is not None else np.zeros((self.n + 31) // 32, dtype=np.uint32)
        n = self._lib.dllm_grammar_build_bitmask_cached(grammar._g, self._v, words.ctypes.data)
        return words, n


def _pieces_callback(pieces):
    """A get_token_str callback over NUL-terminated copies of `pieces` (kept alive by the caller
    through the second return value)."""
    bufs = [None if p is None else C.create_string_buffer(p) for p in pieces]
    addrs = [None if b is None else C.addressof(b) for b in bufs]

    def get(_ctx, i):
        return addrs[i]

    return TOKEN_STR_CB(get), bufs


def lmhead_logits(h, w, *, norm_w=None, eps=1e-6, add_one=False, softcap=0.0, logits=None, stream=None, check=True):
    """Final RMSNorm + logits matvec + softcap (dllm_cuda_lmhead_logits): h fp32 [rows][hidden],
    w [vocab][hidden] fp32 / bf16 / fp16 (CUDA tensors); returns fp32 logits [rows][vocab]."""
    import torch

    rows, hidden = h.shape
    vocab = w.shape[0]
    assert h.dtype == torch.float32 and h.is_contiguous() and w.is_contiguous() and w.shape[1] == hidden
    wdt = {torch.float32: DTYPE_F32, torch.bfloat16: DTYPE_BF16, torch.float16: 2}[w.dtype]
    if logits is None:
        logits = torch.empty(rows, vocab, dtype=torch.float32, device=h.device)
    s = stream if stream is not None else torch.cuda.current_stream(h.device).cuda_stream
    rc = load_library().dllm_cuda_lmhead_logits(rows, hidden, vocab, h.data_ptr(),
                                                None if norm_w is None else norm_w.data_ptr(), float(eps),
                                                int(bool(add_one)), w.data_ptr(), wdt, float(softcap),
                                                logits.data_ptr(), s)
    if check and rc != DLLM_OK:
        raise DllmError(f"dllm_cuda_lmhead_logits: {STATUS_NAMES.get(rc, rc)} "
                        f"({load_library().dllm_cuda_last_error().decode()})")
    return logits
