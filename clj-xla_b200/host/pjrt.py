"""ctypes bindings to a PJRT plugin, call-for-call the same as clj-xla's host.

Mirror of ``src/clj_xla/pjrt.clj``: the PJRT_Api table is read at the same
hard-coded slot offsets (:8-27), every argument struct is a zero-filled byte
block of the same size with fields written at the same byte offsets, named
values use the same 64-byte element stride (:222-259), execute passes one
device, all inputs non-donatable and a 112-byte ExecuteOptions (:454-525), and
events are awaited then destroyed exactly where the reference does.
Errors raise :class:`PJRTError` with the plugin's message (check-error! :63-82).
"""
from __future__ import annotations

import ctypes
import struct
from typing import Dict, List, Optional, Sequence

import numpy as np

# PJRT_Api slot offsets (pjrt.clj:8-27)
OFFSET_API_VERSION = 16
OFFSET_ERROR_DESTROY = 40
OFFSET_ERROR_MESSAGE = 48
OFFSET_ERROR_GET_CODE = 56
OFFSET_PLUGIN_INITIALIZE = 64
OFFSET_PLUGIN_ATTRIBUTES = 72
OFFSET_EVENT_DESTROY = 80
OFFSET_EVENT_AWAIT = 104
OFFSET_CLIENT_CREATE = 120
OFFSET_CLIENT_DESTROY = 128
OFFSET_CLIENT_PLATFORM_NAME = 136
OFFSET_CLIENT_ADDRESSABLE_DEVICES = 168
OFFSET_CLIENT_COMPILE = 200
OFFSET_CLIENT_BUFFER_FROM_HOST_BUFFER = 216
OFFSET_LOADED_EXECUTABLE_DESTROY = 440
OFFSET_LOADED_EXECUTABLE_EXECUTE = 480
OFFSET_BUFFER_DESTROY = 504
OFFSET_BUFFER_TO_HOST_BUFFER = 600

# CompileOptionsProto{executable_build_options{num_replicas=1, num_partitions=1}} (pjrt.clj:32-36)
DEFAULT_COMPILE_OPTIONS_BYTES = bytes([0x1A, 4, 0x20, 1, 0x28, 1])

# PJRT_Buffer_Type codes used by the host (pjrt.clj:400, core.clj:217)
DTYPE_ENUM = {"i8": 2, "i32": 4, "f16": 10, "f32": 11, "bf16": 13}
ELEM_BYTES = {2: 1, 4: 4, 11: 4, 10: 2, 13: 2}

_FN = ctypes.CFUNCTYPE(ctypes.c_void_p, ctypes.c_void_p)
_VFN = ctypes.CFUNCTYPE(None, ctypes.c_void_p)


class PJRTError(RuntimeError):
    def __init__(self, msg: str, code: int = 0):
        super().__init__("PJRT Error: " + msg)
        self.error_msg = msg
        self.code = code


def _w64(buf, off, v):
    struct.pack_into("<Q", buf, off, v & 0xFFFFFFFFFFFFFFFF)


def _w32(buf, off, v):
    struct.pack_into("<i", buf, off, v)


def _r64(buf, off) -> int:
    return struct.unpack_from("<Q", buf, off)[0]


def _addr(buf) -> int:
    return ctypes.addressof(buf)


class PjrtApi:
    """A loaded plugin (``load-plugin!`` pjrt.clj:178-220)."""

    def __init__(self, lib_path: str):
        self.lib = ctypes.CDLL(lib_path, mode=ctypes.RTLD_GLOBAL)
        self._devices = {}
        self._nondon = {}
        get_api = self.lib.GetPjrtApi
        get_api.restype = ctypes.c_void_p
        self.api_ptr = get_api()
        if not self.api_ptr:
            raise PJRTError("GetPjrtApi returned NULL")
        self.api = (ctypes.c_char * 984).from_address(self.api_ptr)  # pjrt.clj:207
        self._fns: Dict[int, object] = {}
        args = ctypes.create_string_buffer(16)
        _w64(args, 0, 16)
        self.check_error(self._call(OFFSET_PLUGIN_INITIALIZE, args))

    def _fn(self, offset: int, void=False):
        key = (offset, void)
        f = self._fns.get(key)
        if f is None:
            ptr = _r64(self.api, offset)
            f = (_VFN if void else _FN)(ptr)
            self._fns[key] = f
        return f

    def _call(self, offset: int, args) -> int:
        return self._fn(offset)(_addr(args)) or 0

    def api_version(self):
        """pjrt.clj:108-114 (reads major from offset 16 - the version struct's size field)."""
        major = struct.unpack_from("<i", self.api, OFFSET_API_VERSION)[0]
        minor = struct.unpack_from("<i", self.api, OFFSET_API_VERSION + 4)[0]
        return major, minor

    def check_error(self, err: int):
        """pjrt.clj:63-82."""
        if not err:
            return
        msg_args = ctypes.create_string_buffer(40)
        _w64(msg_args, 0, 40)
        _w64(msg_args, 16, err)
        self._fn(OFFSET_ERROR_MESSAGE, void=True)(_addr(msg_args))
        sptr, slen = _r64(msg_args, 24), _r64(msg_args, 32)
        msg = ctypes.string_at(sptr, slen).decode("utf-8") if sptr else ""
        code_args = ctypes.create_string_buffer(32)
        _w64(code_args, 0, 32)
        _w64(code_args, 16, err)
        self._call(OFFSET_ERROR_GET_CODE, code_args)
        code = struct.unpack_from("<i", code_args, 24)[0]
        d = ctypes.create_string_buffer(24)
        _w64(d, 0, 24)
        _w64(d, 16, err)
        self._fn(OFFSET_ERROR_DESTROY, void=True)(_addr(d))
        raise PJRTError(msg, code)

    def plugin_attributes(self) -> dict:
        """pjrt.clj:116-146 (64-byte element stride as in the reference)."""
        args = ctypes.create_string_buffer(32)
        _w64(args, 0, 32)
        self.check_error(self._call(OFFSET_PLUGIN_ATTRIBUTES, args))
        ptr, n = _r64(args, 16), _r64(args, 24)
        out = {}
        for i in range(n):
            base = ptr + i * 64
            name_ptr = ctypes.c_uint64.from_address(base + 16).value
            name_len = ctypes.c_uint64.from_address(base + 24).value
            name = ctypes.string_at(name_ptr, name_len).decode()
            vt = ctypes.c_int32.from_address(base + 32).value
            if vt == 0:
                sp = ctypes.c_uint64.from_address(base + 40).value
                sl = ctypes.c_uint64.from_address(base + 48).value
                out[name] = ctypes.string_at(sp, sl).decode()
            elif vt == 1:
                out[name] = ctypes.c_int64.from_address(base + 40).value
        return out

    # ------------------------------------------------------------ events
    def _args24(self):
        """A reusable 24-byte argument struct (struct_size 24, one pointer at
        16) for the per-step Event_Await / Event_Destroy / Buffer_Destroy calls:
        the same bytes the reference writes, without a new allocation per call."""
        a = self.__dict__.get("_a24")
        if a is None:
            a = self._a24 = ctypes.create_string_buffer(24)
            _w64(a, 0, 24)
            self._a24_addr = _addr(a)
        return a

    def _await_destroy(self, event_ptr: int):
        if not event_ptr:
            return
        a = self._args24()
        _w64(a, 16, event_ptr)
        err = self._fn(OFFSET_EVENT_AWAIT)(self._a24_addr) or 0
        _w64(a, 16, event_ptr)
        self._fn(OFFSET_EVENT_DESTROY)(self._a24_addr)
        self.check_error(err)

    # ------------------------------------------------------------ client
    def create_client(self, opts: Optional[dict] = None) -> int:
        """pjrt.clj:222-275 - NamedValues at a 64-byte stride."""
        opts = opts or {}
        args = ctypes.create_string_buffer(88)
        _w64(args, 0, 88)
        keep = []
        if opts:
            nv = ctypes.create_string_buffer(64 * len(opts))
            keep.append(nv)
            for i, (k, v) in enumerate(opts.items()):
                base = i * 64
                kb = ctypes.create_string_buffer(k.encode())
                keep.append(kb)
                _w64(nv, base, 64)
                _w64(nv, base + 16, _addr(kb))
                _w64(nv, base + 24, len(k.encode()))
                if isinstance(v, str):
                    vb = ctypes.create_string_buffer(v.encode())
                    keep.append(vb)
                    _w32(nv, base + 32, 0)
                    _w64(nv, base + 40, _addr(vb))
                    _w64(nv, base + 48, len(v))
                elif isinstance(v, bool):
                    _w32(nv, base + 32, 4)
                    struct.pack_into("<B", nv, base + 40, 1 if v else 0)
                    _w64(nv, base + 48, 1)
                elif isinstance(v, int):
                    _w32(nv, base + 32, 1)
                    struct.pack_into("<q", nv, base + 40, v)
                    _w64(nv, base + 48, 1)
                elif isinstance(v, float):
                    _w32(nv, base + 32, 3)
                    struct.pack_into("<f", nv, base + 40, v)
                    _w64(nv, base + 48, 1)
            _w64(args, 16, _addr(nv))
            _w64(args, 24, len(opts))
        self.check_error(self._call(OFFSET_CLIENT_CREATE, args))
        return _r64(args, 64)

    def destroy_client(self, client: int):
        args = ctypes.create_string_buffer(24)
        _w64(args, 0, 24)
        _w64(args, 16, client)
        self.check_error(self._call(OFFSET_CLIENT_DESTROY, args))

    def platform_name(self, client: int) -> str:
        args = ctypes.create_string_buffer(40)
        _w64(args, 0, 40)
        _w64(args, 16, client)
        self.check_error(self._call(OFFSET_CLIENT_PLATFORM_NAME, args))
        return ctypes.string_at(_r64(args, 24), _r64(args, 32)).decode()

    def addressable_devices(self, client: int) -> List[int]:
        args = ctypes.create_string_buffer(40)
        _w64(args, 0, 40)
        _w64(args, 16, client)
        self.check_error(self._call(OFFSET_CLIENT_ADDRESSABLE_DEVICES, args))
        ptr, n = _r64(args, 24), _r64(args, 32)
        return [ctypes.c_uint64.from_address(ptr + 8 * i).value for i in range(n)]

    def compile_mlir(self, client: int, mlir_text: str) -> int:
        """pjrt.clj:310-340 - format "mlir", 6-byte compile options."""
        code = mlir_text.encode("utf-8")
        code_buf = ctypes.create_string_buffer(code, len(code) + 1)
        fmt = ctypes.create_string_buffer(b"mlir")
        opts = ctypes.create_string_buffer(DEFAULT_COMPILE_OPTIONS_BYTES, len(DEFAULT_COMPILE_OPTIONS_BYTES))
        prog = ctypes.create_string_buffer(48)
        _w64(prog, 0, 48)
        _w64(prog, 16, _addr(code_buf))
        _w64(prog, 24, len(code))
        _w64(prog, 32, _addr(fmt))
        _w64(prog, 40, 4)
        args = ctypes.create_string_buffer(56)
        _w64(args, 0, 56)
        _w64(args, 16, client)
        _w64(args, 24, _addr(prog))
        _w64(args, 32, _addr(opts))
        _w64(args, 40, len(DEFAULT_COMPILE_OPTIONS_BYTES))
        self.check_error(self._call(OFFSET_CLIENT_COMPILE, args))
        return _r64(args, 48)

    def destroy_executable(self, exe: int):
        args = ctypes.create_string_buffer(24)
        _w64(args, 0, 24)
        _w64(args, 16, exe)
        self.check_error(self._call(OFFSET_LOADED_EXECUTABLE_DESTROY, args))

    # ------------------------------------------------------------ buffers
    def buffer_from_host_buffer(self, client: int, host_data: np.ndarray, shape: Sequence[int],
                                dtype_enum: int) -> int:
        """pjrt.clj:342-434 - dense row-major byte strides, semantics=1, await done event."""
        data = np.ascontiguousarray(host_data)
        num_dims = len(shape)
        dims = (ctypes.c_int64 * max(1, num_dims))(*shape)
        args = ctypes.create_string_buffer(120)
        _w64(args, 0, 120)
        _w64(args, 16, client)
        _w64(args, 24, data.ctypes.data if data.size else 0)
        _w32(args, 32, dtype_enum)
        _w64(args, 40, ctypes.addressof(dims))
        _w64(args, 48, num_dims)
        elem = ELEM_BYTES.get(dtype_enum, 4)
        strides = None
        if num_dims > 0:
            strides = (ctypes.c_int64 * num_dims)()
            st = elem
            for i in range(num_dims - 1, -1, -1):
                strides[i] = st
                st *= int(shape[i])
            _w64(args, 56, ctypes.addressof(strides))
            _w64(args, 64, num_dims)
        _w32(args, 72, 1)
        devs = self._devices.get(client)
        if devs is None:  # the device list of a client never changes (pjrt.clj:348-349 takes the first)
            devs = self._devices[client] = self.addressable_devices(client)
        if devs:
            _w64(args, 80, devs[0])
        self.check_error(self._call(OFFSET_CLIENT_BUFFER_FROM_HOST_BUFFER, args))
        done, buf = _r64(args, 104), _r64(args, 112)
        self._await_destroy(done)
        return buf

    def destroy_buffer(self, buf: int):
        if not buf:
            return
        a = self._args24()
        _w64(a, 16, buf)
        err = self._fn(OFFSET_BUFFER_DESTROY)(self._a24_addr)
        if err:
            self.check_error(err)

    def execute_executable(self, exe: int, input_buffers: Sequence[int], num_outputs: int = 1,
                           wait: bool = True):
        """pjrt.clj:454-525.  ``wait=False`` skips awaiting the completion event
        (destroyed unawaited; the library's stream keeps execution ordered) so
        a caller can enqueue several steps back to back."""
        n = len(input_buffers)
        nouts = max(1, int(num_outputs))
        # the argument list as one uint64 array (numpy: a few µs for the ~500
        # buffers of a decode step, where a ctypes array built from a list costs
        # 150 µs)
        arg_ptrs = np.fromiter(input_buffers, dtype=np.uint64, count=n) if n else np.zeros(1, np.uint64)
        if n and not arg_ptrs.all():
            raise PJRTError(f"NULL input buffer {int(np.flatnonzero(arg_ptrs == 0)[0])}")
        arg_lists = (ctypes.c_uint64 * 1)(arg_ptrs.ctypes.data)
        out_ptrs = (ctypes.c_uint64 * nouts)()
        out_lists = (ctypes.c_uint64 * 1)(ctypes.addressof(out_ptrs))
        events = (ctypes.c_uint64 * 1)()
        nondon = self._nondon.get(n)  # every input index (pjrt.clj:478-480); the same array per count
        if nondon is None:
            nondon = self._nondon[n] = (ctypes.c_int64 * max(1, n))(*range(n))
        opts = ctypes.create_string_buffer(144)
        _w64(opts, 0, 112)
        _w64(opts, 56, ctypes.addressof(nondon))
        _w64(opts, 64, n)
        args = ctypes.create_string_buffer(80)
        _w64(args, 0, 80)
        _w64(args, 16, exe)
        _w64(args, 24, _addr(opts))
        _w64(args, 32, ctypes.addressof(arg_lists))
        _w64(args, 40, 1)
        _w64(args, 48, n)
        _w64(args, 56, ctypes.addressof(out_lists))
        _w64(args, 64, ctypes.addressof(events))
        self.check_error(self._call(OFFSET_LOADED_EXECUTABLE_EXECUTE, args))
        if wait:
            self._await_destroy(events[0])
        elif events[0]:
            d = ctypes.create_string_buffer(24)
            _w64(d, 0, 24)
            _w64(d, 16, events[0])
            self._call(OFFSET_EVENT_DESTROY, d)
        if nouts == 1:
            return out_ptrs[0]
        return list(out_ptrs)

    def buffer_to_host(self, buf: int, nbytes: int, out: Optional[np.ndarray] = None) -> np.ndarray:
        """pjrt.clj:527-563 (dst_size given by the caller; the reference passes numel*4)."""
        dst = out if out is not None else np.empty(nbytes, np.uint8)
        args = ctypes.create_string_buffer(56)
        _w64(args, 0, 56)
        _w64(args, 16, buf)
        _w64(args, 24, 0)
        _w64(args, 32, dst.ctypes.data)
        _w64(args, 40, dst.nbytes)
        self.check_error(self._call(OFFSET_BUFFER_TO_HOST_BUFFER, args))
        self._await_destroy(_r64(args, 48))
        return dst

    def buffer_to_host_floats(self, buf: int, num_floats: int) -> np.ndarray:
        """``buffer-to-host-buffer`` pjrt.clj:527-563 - reads num_floats f32 values."""
        a = np.zeros(num_floats, np.float32)
        self.buffer_to_host(buf, num_floats * 4, a)
        return a
