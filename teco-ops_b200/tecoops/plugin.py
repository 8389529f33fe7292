"""Drive the inference plugins (libteco_ops_plugin.so) the way the Teco-Inference
engine does: shape inference, then Enqueue on a stream with named inputs.

The plugins follow reference teco/plugin/plugin*/plugin_*.cc; the engine itself
is not available here, so this module plays its part through the stand-in
plugin host's C entry points.
"""
from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
PLUGIN_PATH = os.path.join(_HERE, "libteco_ops_plugin.so")
_lib = None


def lib():
    global _lib
    if _lib is None:
        from . import capi
        capi.lib()   # libteco_ops.so first (the plugin library links it)
        L = ctypes.CDLL(PLUGIN_PATH)
        L.teco_plugin_last_error.restype = ctypes.c_char_p
        _lib = L
    return _lib


def registered() -> dict:
    buf = ctypes.create_string_buffer(4096)
    lib().teco_plugin_list(buf, 4096)
    out = {}
    for item in buf.value.decode().split(";"):
        if item:
            name, ins = item.split(":")
            out[name] = ins.split(",") if ins else []
    return out


def _attrs(attrs: dict):
    names = (ctypes.c_char_p * len(attrs))(*[k.encode() for k in attrs])
    vals = (ctypes.c_double * len(attrs))(*[float(v) for v in attrs.values()])
    return len(attrs), names, vals


def _shapes(shapes):
    ranks = (ctypes.c_int * len(shapes))(*[len(s) for s in shapes])
    flat = [int(d) for s in shapes for d in s]
    dims = (ctypes.c_int * max(1, len(flat)))(*flat)
    return ranks, dims


def infer_output_shape(op: str, input_shapes, attrs: dict, n_out: int = 1):
    """Shape of output 0 (n_out == 1) or the list of the n_out output shapes."""
    ranks, dims = _shapes(input_shapes)
    na, names, vals = _attrs(attrs)
    out_ranks = (ctypes.c_int * n_out)()
    out_dims = (ctypes.c_int * (8 * n_out))()
    st = lib().teco_plugin_infer(op.encode(), len(input_shapes), ranks, dims, na, names, vals,
                                 n_out, out_ranks, out_dims)
    if st != 0:
        raise RuntimeError(f"{op}: infer failed ({st}): {lib().teco_plugin_last_error().decode()}")
    shapes = [list(out_dims)[8 * o:8 * o + out_ranks[o]] for o in range(n_out)]
    return shapes[0] if n_out == 1 else shapes


def enqueue(op: str, inputs: dict, outputs, attrs: dict, stream: int = 0):
    """inputs: name -> (device pointer, shape); outputs: list of device pointers."""
    names = list(inputs)
    in_names = (ctypes.c_char_p * len(names))(*[n.encode() for n in names])
    in_ptrs = (ctypes.c_void_p * len(names))(*[inputs[n][0] for n in names])
    ranks, dims = _shapes([inputs[n][1] for n in names])
    out_ptrs = (ctypes.c_void_p * len(outputs))(*outputs)
    na, an, av = _attrs(attrs)
    st = lib().teco_plugin_enqueue(op.encode(), len(names), in_names, in_ptrs, ranks, dims,
                                   len(outputs), out_ptrs, na, an, av, ctypes.c_void_p(stream))
    if st != 0:
        raise RuntimeError(f"{op}: enqueue failed ({st}): {lib().teco_plugin_last_error().decode()}")


class Instance:
    """A plugin op instance that lives across Enqueue calls, as an engine keeps one per
    graph node (its device buffers and tecoops handle are reused)."""

    def __init__(self, op: str):
        self.id = lib().teco_plugin_create(op.encode())
        if self.id < 0:
            raise RuntimeError(f"{op}: unknown plugin op")
        self.op = op

    def enqueue(self, inputs: dict, outputs, attrs: dict, stream: int = 0):
        names = list(inputs)
        in_names = (ctypes.c_char_p * len(names))(*[n.encode() for n in names])
        in_ptrs = (ctypes.c_void_p * len(names))(*[inputs[n][0] for n in names])
        ranks, dims = _shapes([inputs[n][1] for n in names])
        out_ptrs = (ctypes.c_void_p * len(outputs))(*outputs)
        na, an, av = _attrs(attrs)
        st = lib().teco_plugin_enqueue_instance(self.id, len(names), in_names, in_ptrs, ranks,
                                                dims, len(outputs), out_ptrs, na, an, av,
                                                ctypes.c_void_p(stream))
        if st != 0:
            raise RuntimeError(f"{self.op}: enqueue failed ({st}): "
                               f"{lib().teco_plugin_last_error().decode()}")

    def close(self):
        if self.id > 0:
            lib().teco_plugin_destroy(self.id)
            self.id = -1
