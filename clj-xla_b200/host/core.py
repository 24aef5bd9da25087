"""High-level host API: init / compile-graph / execute / to-host-slice.

Mirror of ``src/clj_xla/core.clj`` (``init-backend!`` :129-167, ``compile-graph``
:179-187, ``buffer-from-host-buffer`` :189-195, ``execute`` :197-223,
``to-host-slice`` :225-242, ``destroy-buffer!`` :244-249) and of the SHA-256
executable cache in ``src/clj_xla/compile.clj:13-29``.  The B200 library is
selected the way the reference selects any plugin: by passing its path as the
backend target (core.clj:146-147).
"""
from __future__ import annotations

import ctypes
import hashlib
import os
from typing import Dict, List, Optional, Sequence

import numpy as np

from .pjrt import DTYPE_ENUM, PjrtApi
from .stablehlo import graph_to_mlir_text

_DEFAULT_CONTEXT = None
_EXEC_CACHE: Dict[tuple, dict] = {}


def default_library_path() -> str:
    from .. import LIB_PATH  # type: ignore
    return os.environ.get("CLJXLA_B200_LIBRARY_PATH", LIB_PATH)


class Context(dict):
    pass


def init_backend(target: Optional[str] = None, client_opts: Optional[dict] = None) -> Context:
    """core.clj:129-167 - load the plugin at ``target`` (a path), create a client."""
    global _DEFAULT_CONTEXT
    lib_path = target or default_library_path()
    if not os.path.exists(lib_path):
        raise FileNotFoundError(f"PJRT plugin not found: {lib_path} (build it with clj-xla_b200/build.py)")
    api = PjrtApi(lib_path)
    client = api.create_client({"allocator": "platform"} if client_opts is None else client_opts)
    ctx = Context(api=api, client=client, platform=api.platform_name(client), target=lib_path)
    _DEFAULT_CONTEXT = ctx
    return ctx


def get_context() -> Context:
    if _DEFAULT_CONTEXT is None:
        return init_backend()
    return _DEFAULT_CONTEXT


def _sha256(s: str) -> str:
    return hashlib.sha256(s.encode("utf-8")).hexdigest()


def compile_graph(ctx: Context, graph: dict) -> dict:
    """compile.clj:13-24 - MLIR text -> SHA-256 -> cached executable."""
    text = graph_to_mlir_text(graph)
    return compile_mlir_text(ctx, text, graph)


def compile_mlir_text(ctx: Context, text: str, graph: Optional[dict] = None) -> dict:
    key = (ctx["client"], _sha256(text))
    hit = _EXEC_CACHE.get(key)
    if hit is not None:
        return dict(hit, graph=graph)
    handle = ctx["api"].compile_mlir(ctx["client"], text)
    exe = {"handle": handle, "hash": key, "graph": graph, "ctx": ctx, "text": text}
    _EXEC_CACHE[key] = exe
    return exe


def clear_cache():
    """compile.clj:26-29."""
    _EXEC_CACHE.clear()


def close_backend(ctx: Context):
    """Destroys the client's cached executables and then the client (a
    tensor-parallel client also leaves its NCCL group)."""
    global _DEFAULT_CONTEXT
    for key in [k for k in _EXEC_CACHE if k[0] == ctx["client"]]:
        ctx["api"].destroy_executable(_EXEC_CACHE.pop(key)["handle"])
    ctx["api"].destroy_client(ctx["client"])
    if _DEFAULT_CONTEXT is ctx:
        _DEFAULT_CONTEXT = None


def buffer_from_host_buffer(ctx: Context, host_data: np.ndarray, shape: Sequence[int], dtype_enum: int) -> int:
    return ctx["api"].buffer_from_host_buffer(ctx["client"], host_data, list(shape), dtype_enum)


def execute(exe: dict, inputs: Sequence) -> List[int]:
    """core.clj:197-223 - host arrays are uploaded with the invar dtypes first."""
    ctx = exe["ctx"]
    graph = exe.get("graph")
    n_out = len(graph["outvars"]) if graph else None
    bufs = []
    for i, x in enumerate(inputs):
        if isinstance(x, int):
            bufs.append(x)
        else:
            _, (_, shape, dt) = graph["invars"][i]
            bufs.append(buffer_from_host_buffer(ctx, np.asarray(x), shape, DTYPE_ENUM[dt]))
    if n_out is None:
        n_out = 1
    out = ctx["api"].execute_executable(exe["handle"], bufs, n_out)
    return out if isinstance(out, list) else [out]


def to_host_slice(ctx: Context, out_buf: int, slice_idx: int, vocab_size: int, total_elements: int) -> np.ndarray:
    """core.clj:225-242 - copy total floats, return row ``slice_idx``."""
    n = max(int(total_elements), (slice_idx + 1) * vocab_size)
    allf = ctx["api"].buffer_to_host_floats(out_buf, n)
    off = slice_idx * vocab_size
    if 0 <= off and off + vocab_size <= allf.size:
        return allf[off:off + vocab_size].copy()
    return allf


def destroy_buffer(ctx: Context, buf: int):
    try:
        ctx["api"].destroy_buffer(buf)
    except Exception:
        pass


def buffer_to_numpy(ctx: Context, buf: int, shape: Sequence[int], dt: str) -> np.ndarray:
    """Typed read-back (f32 / i32 / bf16 bits as uint16)."""
    np_dt = {"f32": np.float32, "i32": np.int32, "bf16": np.uint16, "f16": np.float16, "i8": np.int8}[dt]
    n = int(np.prod(shape)) if len(shape) else 1
    a = np.empty(n, np_dt)
    ctx["api"].buffer_to_host(buf, a.nbytes, a.view(np.uint8))
    return a.reshape(shape)


# ------------------------------------------------------------ library extras
def _lib(ctx: Context):
    return ctx["api"].lib


def kernel_launches(ctx: Context) -> int:
    f = _lib(ctx).cljxla_b200_kernel_launches
    f.restype = ctypes.c_int64
    return int(f())


def plan_info(ctx: Context, exe: dict) -> dict:
    f = _lib(ctx).cljxla_b200_plan_info
    f.argtypes = [ctypes.c_void_p, ctypes.POINTER(ctypes.c_int64), ctypes.c_int]
    info = (ctypes.c_int64 * 8)()
    f(ctypes.c_void_p(exe["handle"]), info, 8)
    keys = ["launches", "arena_bytes", "nodes", "live_nodes", "fused_groups", "const_bytes", "jit_missing",
            "computed_masks"]
    return dict(zip(keys, list(info)))


def profile_enable(ctx: Context, on: bool):
    f = _lib(ctx).cljxla_b200_profile_enable
    f.argtypes = [ctypes.c_int]
    f(1 if on else 0)


def profile_dump(ctx: Context):
    import json
    f = _lib(ctx).cljxla_b200_profile_dump
    f.argtypes = [ctypes.c_char_p, ctypes.c_size_t]
    f.restype = ctypes.c_size_t
    n = f(None, 0)
    buf = ctypes.create_string_buffer(n + 16)
    f(buf, n + 16)
    return json.loads(buf.value.decode())


def client_stream(ctx: Context) -> int:
    f = _lib(ctx).cljxla_b200_stream
    f.argtypes = [ctypes.c_void_p]
    f.restype = ctypes.c_void_p
    return f(ctypes.c_void_p(ctx["client"])) or 0


def nccl_unique_id(lib_path: Optional[str] = None) -> str:
    """Hex NCCL unique id for a tensor-parallel group (made on one rank, passed
    to every rank's client as ``tp_nccl_id``).  Needs no device."""
    lib = ctypes.CDLL(lib_path or default_library_path())
    f = lib.cljxla_b200_nccl_unique_id
    f.argtypes = [ctypes.c_char_p, ctypes.c_size_t]
    f.restype = ctypes.c_int
    buf = ctypes.create_string_buffer(512)
    rc = f(buf, 512)
    if rc != 0:
        raise RuntimeError(f"cljxla_b200_nccl_unique_id failed ({rc})")
    return buf.value.decode()


def init_tp_backend(tp_size: int, tp_rank: int, nccl_id: str, device: Optional[int] = None,
                    target: Optional[str] = None) -> Context:
    """A client that is rank ``tp_rank`` of a ``tp_size``-way tensor-parallel
    group: every rank calls this with the same ``nccl_id`` (collective)."""
    opts = {"allocator": "platform", "tp_size": int(tp_size), "tp_rank": int(tp_rank), "tp_nccl_id": nccl_id}
    if device is not None:
        opts["device"] = int(device)
    return init_backend(target, opts)


def p2p_export(ctx: Context, slot_bytes: int = 32 << 10) -> str:
    """This rank's exchange-buffer handle for the one-shot peer all-reduce."""
    f = _lib(ctx).cljxla_b200_p2p_export
    f.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_char_p, ctypes.c_size_t]
    f.restype = ctypes.c_int
    out = ctypes.create_string_buffer(256)
    rc = f(ctypes.c_void_p(ctx["client"]), int(slot_bytes), out, 256)
    if rc != 0:
        raise RuntimeError(f"cljxla_b200_p2p_export failed ({rc})")
    return out.value.decode()


def p2p_import(ctx: Context, handles: Sequence[str]):
    """Maps every rank's exchange buffer (handles in rank order); from here on
    small all_reduce ops run as the one-shot peer kernel."""
    f = _lib(ctx).cljxla_b200_p2p_import
    f.argtypes = [ctypes.c_void_p, ctypes.c_char_p, ctypes.c_size_t]
    f.restype = ctypes.c_int
    b = "".join(handles).encode()
    rc = f(ctypes.c_void_p(ctx["client"]), b, len(b))
    if rc != 0:
        raise RuntimeError(f"cljxla_b200_p2p_import failed ({rc})")


def plan_text(lib_path: str, text: str, fuse: bool = True) -> dict:
    """Host-only parse+plan through the library (no device needed)."""
    lib = ctypes.CDLL(lib_path)
    f = lib.cljxla_b200_plan_text
    f.argtypes = [ctypes.c_char_p, ctypes.c_size_t, ctypes.c_int, ctypes.POINTER(ctypes.c_int64), ctypes.c_int,
                  ctypes.c_char_p, ctypes.c_size_t]
    f.restype = ctypes.c_int
    b = text.encode()
    info = (ctypes.c_int64 * 8)()
    err = ctypes.create_string_buffer(4096)
    flags = int(fuse) if not isinstance(fuse, bool) else (1 if fuse else 0)  # bit 0 fusion, bit 1 in-place KV
    rc = f(b, len(b), flags, info, 8, err, 4096)
    if rc != 0:
        raise RuntimeError(f"plan failed ({rc}): {err.value.decode()}")
    keys = ["launches", "arena_bytes", "nodes", "live_nodes", "fused_groups", "const_bytes", "jit_missing",
            "computed_masks"]
    return dict(zip(keys, list(info)))
