"""A minimal XLA FFI host in ctypes, for driving the handler library in tests.

It plays the part XLA's runtime plays for a registered custom call: it builds
XLA_FFI_CallFrame structures (XLA FFI C API 0.4, the jaxlib 0.11.2 headers),
supplies the few API entries the handlers use (error create / details /
destroy, stream get, state set / get), registers the prepared-state type ids
and deletes prepared states through their type info, as
``jax.ffi.register_ffi_type`` and an executable's teardown do.
"""

from __future__ import annotations

import ctypes
from ctypes import POINTER, c_char_p, c_int, c_int64, c_size_t, c_void_p

# XLA_FFI_DataType / ArgType / RetType / AttrType / ExecutionStage / Error_Code.
S32, S64, F32, F64, C64, C128 = 4, 5, 11, 12, 15, 18
ARG_BUFFER = RET_BUFFER = 1
ATTR_ARRAY, ATTR_SCALAR = 1, 3
INSTANTIATE, EXECUTE = 0, 3
ERROR_NAMES = {3: "INVALID_ARGUMENT", 13: "INTERNAL", 9: "FAILED_PRECONDITION"}

_TORCH_CODES = {"torch.int32": S32, "torch.int64": S64, "torch.float32": F32, "torch.float64": F64,
                "torch.complex64": C64, "torch.complex128": C128}


class ByteSpan(ctypes.Structure):
    _fields_ = [("ptr", c_char_p), ("len", c_size_t)]


class Array(ctypes.Structure):
    _fields_ = [("dtype", c_int), ("size", c_size_t), ("data", c_void_p)]


class Scalar(ctypes.Structure):
    _fields_ = [("dtype", c_int), ("value", c_void_p)]


class Buffer(ctypes.Structure):
    _fields_ = [("struct_size", c_size_t), ("extension_start", c_void_p), ("dtype", c_int),
                ("data", c_void_p), ("rank", c_int64), ("dims", POINTER(c_int64))]


class _List(ctypes.Structure):
    _fields_ = [("struct_size", c_size_t), ("extension_start", c_void_p), ("size", c_int64),
                ("types", POINTER(c_int)), ("items", POINTER(c_void_p))]


class Attrs(ctypes.Structure):
    _fields_ = [("struct_size", c_size_t), ("extension_start", c_void_p), ("size", c_int64),
                ("types", POINTER(c_int)), ("names", POINTER(c_void_p)), ("attrs", POINTER(c_void_p))]


class ApiVersion(ctypes.Structure):
    _fields_ = [("struct_size", c_size_t), ("extension_start", c_void_p), ("major_version", c_int),
                ("minor_version", c_int)]


_API_ENTRIES = ("Error_Create", "Error_GetDetails", "Error_Destroy", "Handler_Register", "Stream_Get",
                "Type_Register", "InvokeContext_Get", "State_Set", "State_Get", "DeviceMemory_Allocate",
                "DeviceMemory_Free", "ThreadPool_Schedule", "ThreadPool_NumThreads", "Future_Create",
                "Future_SetAvailable", "Future_SetError", "RunId_Get", "DeviceOrdinal_Get",
                "InvokeContext_FindExtension")


class Api(ctypes.Structure):
    _fields_ = [("struct_size", c_size_t), ("extension_start", c_void_p), ("api_version", ApiVersion),
                ("internal_api", c_void_p)] + [(name, c_void_p) for name in _API_ENTRIES]


class CallFrame(ctypes.Structure):
    _fields_ = [("struct_size", c_size_t), ("extension_start", c_void_p), ("api", POINTER(Api)),
                ("ctx", c_void_p), ("stage", c_int), ("args", _List), ("rets", _List), ("attrs", Attrs),
                ("future", c_void_p)]


class ErrorCreateArgs(ctypes.Structure):
    _fields_ = [("struct_size", c_size_t), ("extension_start", c_void_p), ("message", c_char_p), ("errc", c_int)]


class ErrorGetDetailsArgs(ctypes.Structure):
    _fields_ = [("struct_size", c_size_t), ("extension_start", c_void_p), ("error", c_void_p),
                ("message", c_char_p), ("errc", c_int)]


class ErrorDestroyArgs(ctypes.Structure):
    _fields_ = [("struct_size", c_size_t), ("extension_start", c_void_p), ("error", c_void_p)]


class StreamGetArgs(ctypes.Structure):
    _fields_ = [("struct_size", c_size_t), ("extension_start", c_void_p), ("ctx", c_void_p), ("stream", c_void_p)]


class StateArgs(ctypes.Structure):
    _fields_ = [("struct_size", c_size_t), ("extension_start", c_void_p), ("ctx", c_void_p), ("stage", c_int),
                ("type_id", POINTER(c_int64)), ("state", c_void_p)]


class TypeInfo(ctypes.Structure):
    _fields_ = [("struct_size", c_size_t), ("extension_start", c_void_p), ("deleter", c_void_p)]


_ENTRY = ctypes.CFUNCTYPE(c_void_p, c_void_p)
_HANDLER = ctypes.CFUNCTYPE(c_void_p, POINTER(CallFrame))


class HandlerError(RuntimeError):
    def __init__(self, code: int, message: str):
        super().__init__(f"{ERROR_NAMES.get(code, code)}: {message}")
        self.code = code
        self.message = message


class Host:
    """One XLA-like runtime: an API table, states per call site, one stream."""

    def __init__(self, library: ctypes.CDLL, registration: dict[str, int], stream: int = 0):
        self.library = library
        self.registration = registration
        self.stream = stream
        self._errors: dict[int, tuple[int, bytes]] = {}
        self._next_error = 1
        self._states: dict[int, dict[int, int]] = {}   # ctx -> type id -> state
        self._callbacks = {
            "Error_Create": _ENTRY(self._error_create),
            "Error_GetDetails": _ENTRY(self._error_details),
            "Error_Destroy": _ENTRY(self._error_destroy),
            "Stream_Get": _ENTRY(self._stream_get),
            "State_Set": _ENTRY(self._state_set),
            "State_Get": _ENTRY(self._state_get),
        }
        self.api = Api()
        self.api.struct_size = ctypes.sizeof(Api)
        self.api.api_version = ApiVersion(ctypes.sizeof(ApiVersion), None, 0, 4)
        for name, callback in self._callbacks.items():
            setattr(self.api, name, ctypes.cast(callback, c_void_p).value)
        # Register the prepared-state type ids (jax.ffi.register_ffi_type).
        self.type_ids = {}
        for index, operation in enumerate(("copy", "update", "dot", "accumulation", "reduction"), start=1):
            pointer = ctypes.cast(registration[f"{operation}_type_id"], POINTER(c_int64))
            pointer[0] = 100 + index
            self.type_ids[operation] = 100 + index
        self._next_ctx = 1

    # -- API entries ---------------------------------------------------------
    def _error_create(self, address):
        args = ErrorCreateArgs.from_address(address)
        handle = self._next_error
        self._next_error += 1
        self._errors[handle] = (args.errc, args.message or b"")
        return handle

    def _error_details(self, address):
        args = ErrorGetDetailsArgs.from_address(address)
        code, message = self._errors[args.error]
        args.errc = code
        args.message = message
        return None

    def _error_destroy(self, address):
        self._errors.pop(ErrorDestroyArgs.from_address(address).error, None)
        return None

    def _stream_get(self, address):
        StreamGetArgs.from_address(address).stream = self.stream
        return None

    def _state_set(self, address):
        args = StateArgs.from_address(address)
        self._states.setdefault(args.ctx, {})[args.type_id[0]] = args.state
        return None

    def _state_get(self, address):
        args = StateArgs.from_address(address)
        state = self._states.get(args.ctx, {}).get(args.type_id[0])
        if state is None:
            return self._error_create(ctypes.addressof(ErrorCreateArgs(0, None, b"state not found", 9)))
        args.state = state
        return None

    # -- call frames ---------------------------------------------------------
    def _raise(self, handle):
        if handle:
            code, message = self._errors.pop(handle)
            raise HandlerError(code, message.decode())

    def _frame(self, ctx, stage, args, rets, attrs):
        keep = []

        def buffers(items, kind):
            types = (c_int * max(len(items), 1))(*([kind] * len(items)))
            pointers = (c_void_p * max(len(items), 1))()
            for i, (code, data, dims) in enumerate(items):
                shape = (c_int64 * max(len(dims), 1))(*dims)
                buffer = Buffer(ctypes.sizeof(Buffer), None, code, data, len(dims), shape)
                keep.extend((shape, buffer))
                pointers[i] = ctypes.addressof(buffer)
            keep.extend((types, pointers))
            return _List(ctypes.sizeof(_List), None, len(items), types, pointers)

        names = sorted(attrs)   # XLA passes attributes sorted by name
        attr_types = (c_int * max(len(names), 1))()
        attr_names = (c_void_p * max(len(names), 1))()
        attr_values = (c_void_p * max(len(names), 1))()
        for i, name in enumerate(names):
            raw = name.encode()
            span = ByteSpan(raw, len(raw))
            value = attrs[name]
            if isinstance(value, int):
                cell = c_int64(value)
                item = Scalar(S64, ctypes.addressof(cell))
                attr_types[i] = ATTR_SCALAR
                keep.append(cell)
            else:
                data = (c_int64 * max(len(value), 1))(*[int(v) for v in value])
                item = Array(S64, len(value), ctypes.addressof(data))
                attr_types[i] = ATTR_ARRAY
                keep.append(data)
            keep.extend((raw, span, item))
            attr_names[i] = ctypes.addressof(span)
            attr_values[i] = ctypes.addressof(item)
        keep.extend((attr_types, attr_names, attr_values))
        frame = CallFrame()
        frame.struct_size = CallFrame.future.offset   # XLA_FFI_CallFrame_STRUCT_SIZE ends at attrs
        frame.api = ctypes.pointer(self.api)
        frame.ctx = ctx
        frame.stage = stage
        frame.args = buffers(args, ARG_BUFFER)
        frame.rets = buffers(rets, RET_BUFFER)
        frame.attrs = Attrs(ctypes.sizeof(Attrs), None, len(names), attr_types, attr_names, attr_values)
        return frame, keep

    def instantiate(self, operation: str, **attrs) -> int:
        """Run the operation's instantiate handler; returns the call-site context."""
        ctx = self._next_ctx
        self._next_ctx += 1
        frame, keep = self._frame(ctx, INSTANTIATE, [], [], attrs)
        handler = _HANDLER(self.registration[f"{operation}_instantiate"])
        self._raise(handler(ctypes.byref(frame)))
        del keep
        return ctx

    def execute(self, operation: str, suffix: str, ctx: int, args, rets) -> None:
        """Run an execute handler; args / rets are (tensor or (code, address, dims))."""
        frame, keep = self._frame(ctx, EXECUTE, [_describe(a) for a in args], [_describe(r) for r in rets], {})
        handler = _HANDLER(self.registration[f"{operation}_{suffix}"])
        self._raise(handler(ctypes.byref(frame)))
        del keep

    def destroy(self, operation: str, ctx: int) -> None:
        """Delete the call site's prepared state through the type's deleter."""
        state = self._states.get(ctx, {}).pop(self.type_ids[operation], None)
        if state is not None:
            info = TypeInfo.from_address(self.registration[f"{operation}_type_info"])
            ctypes.CFUNCTYPE(None, c_void_p)(info.deleter)(state)


def _describe(value):
    if isinstance(value, tuple):
        return value
    return (_TORCH_CODES[str(value.dtype)], value.data_ptr(), tuple(value.shape))
