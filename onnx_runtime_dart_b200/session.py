"""Host mirror of the reference's operator interface for the matmul hot path.

The reference dispatches nodes in ``OnnxGraphExecutor._dispatch``
(lib/src/onnx_graph.dart:961) and keeps weights in ``_initializers`` plus
prepacked Gemm B in ``_prepackedGemmB`` (:51-56).  ``CudaSession`` is the
B200 counterpart for the three hot ops: weights are uploaded once (keyed
by initializer name), activations may stay on the device between ops
(``DeviceTensor``), and ``dispatch`` mirrors the ``'MatMul'``, ``'Gemm'``
and ``'MatMulNBits'`` cases (:1154-1173, :1584-1596) including their
error behaviour.  The module-level ``op_*`` functions mirror the pure op
functions (``opMatMulNBits`` onnx_qlinear_ops.dart:114-156, ``opGemm``
onnx_ops.dart:1777-1793, ``opMatMul`` :1375-1431) on a throwaway session.

Every compute call goes through libort_cuda.so (CUDA, sm_100a); nothing in
this module computes a matmul on the CPU.
"""
from __future__ import annotations

import ctypes
import os
from typing import Dict, List, Optional, Sequence, Tuple, Union

import numpy as np

from . import _lib
from ._lib import StateError, UnsupportedError, check


def _ptr(a) -> int:
    """Address of a numpy array, a torch CUDA tensor or a DeviceTensor."""
    if a is None:
        return 0
    if isinstance(a, DeviceTensor):
        return a.ptr
    if isinstance(a, np.ndarray):
        return a.ctypes.data
    if hasattr(a, "data_ptr"):
        return int(a.data_ptr())
    raise TypeError(f"unsupported buffer type {type(a)}")


class DeviceTensor:
    """An fp32 activation resident in the session's device memory."""

    def __init__(self, session: "CudaSession", shape: Sequence[int], ptr: Optional[int] = None):
        self.session = session
        self.shape = tuple(int(d) for d in shape)
        self.nbytes = int(np.prod(self.shape, dtype=np.int64)) * 4 if self.shape else 4
        if ptr is None:
            p = ctypes.c_void_p()
            check(_lib.load().ort_cuda_alloc(session.handle, self.nbytes, ctypes.byref(p)),
                  "ort_cuda_alloc")
            self.ptr = p.value or 0
            self._owned = True
        else:
            self.ptr = ptr
            self._owned = False

    @classmethod
    def from_host(cls, session: "CudaSession", a: np.ndarray) -> "DeviceTensor":
        a = np.ascontiguousarray(a, dtype=np.float32)
        t = cls(session, a.shape)
        check(_lib.load().ort_cuda_h2d(session.handle, t.ptr, a.ctypes.data, a.nbytes),
              "ort_cuda_h2d")
        return t

    def numpy(self) -> np.ndarray:
        out = np.empty(self.shape, np.float32)
        check(_lib.load().ort_cuda_d2h(self.session.handle, out.ctypes.data, self.ptr,
                                       self.nbytes), "ort_cuda_d2h")
        return out

    def free(self) -> None:
        if self._owned and self.ptr and self.session.handle:
            check(_lib.load().ort_cuda_free(self.session.handle, self.ptr), "ort_cuda_free")
        self.ptr = 0

    @property
    def rank(self) -> int:
        return len(self.shape)


Tensorish = Union[np.ndarray, DeviceTensor]


class CudaSession:
    """One GPU (or one rank of an N-sharded group) running the hot ops.

    mode: "exact" (fp32 FFMA), "strict" (bitwise reference rounding),
    "mma_f16" / "mma_bf16" (tcgen05 tensor cores)."""

    def __init__(self, device: int = 0, mode: str = "exact", rank: int = 0, world: int = 1,
                 nccl_id: Optional[bytes] = None, timeout_ms: int = 60000):
        L = _lib.load()
        h = ctypes.c_void_p()
        m = _lib.MODES[mode]
        if world == 1:
            check(L.ort_cuda_open(device, m, ctypes.byref(h)), "ort_cuda_open")
        else:
            if nccl_id is None or len(nccl_id) != 128:
                raise ValueError("a 128-byte NCCL unique id is required for world > 1")
            buf = ctypes.create_string_buffer(nccl_id, 128)
            check(L.ort_cuda_open_rank(device, rank, world, buf, m, timeout_ms, ctypes.byref(h)),
                  "ort_cuda_open_rank")
        self.handle = h.value
        self.device, self.rank, self.world, self.mode = device, rank, world, mode
        # initializer name -> ("nbits" | "dense", K, N)
        self.weights: Dict[str, tuple] = {}
        self._explicit_stream = False  # set_stream() chose the launch stream
        self._followed: Optional[int] = None

    @staticmethod
    def nccl_unique_id() -> bytes:
        buf = ctypes.create_string_buffer(128)
        check(_lib.load().ort_cuda_nccl_unique_id(buf), "ort_cuda_nccl_unique_id")
        return buf.raw

    # -- lifecycle -------------------------------------------------------
    def close(self) -> None:
        if self.handle:
            check(_lib.load().ort_cuda_close(self.handle), "ort_cuda_close")
            self.handle = None

    dispose = close  # OnnxModel.dispose (lib/onnx_runtime_dart.dart:140)

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def set_mode(self, mode: str) -> None:
        check(_lib.load().ort_cuda_set_mode(self.handle, _lib.MODES[mode]), "ort_cuda_set_mode")
        self.mode = mode

    def set_stream(self, stream_ptr: Optional[int]) -> None:
        """Launch on an existing cudaStream_t.  0 is the legacy default
        stream (torch's default stream), passed as cudaStreamLegacy; None
        restores the session's own stream."""
        self._explicit_stream = stream_ptr is not None
        self._followed = None
        self._set_stream_raw(stream_ptr)

    def _set_stream_raw(self, stream_ptr: Optional[int]) -> None:
        if stream_ptr is None:
            arg = None
        else:
            arg = stream_ptr if stream_ptr else 1  # cudaStreamLegacy == (cudaStream_t)0x1
        check(_lib.load().ort_cuda_set_stream(self.handle, arg), "ort_cuda_set_stream")

    def _follow_torch_stream(self) -> None:
        """Calls on torch CUDA tensors launch on torch's current stream
        (unless set_stream() chose one), so they are ordered after the
        kernels that produced their inputs and before those that read their
        outputs, as torch ops are."""
        if self._explicit_stream:
            return
        import torch
        cur = torch.cuda.current_stream().cuda_stream
        if cur != self._followed:
            self._set_stream_raw(cur)
            self._followed = cur

    def set_peer_wait(self, ms: int) -> None:
        """Bound of every wait for a peer GPU in the exchange of Y (ms)."""
        check(_lib.load().ort_cuda_set_peer_wait(self.handle, int(ms)), "ort_cuda_set_peer_wait")

    def set_replicate_bytes(self, nbytes: int) -> None:
        """MatMulNBits weights of at most nbytes packed bytes uploaded from now
        on are kept whole on every rank (no exchange); -1: the default
        (10 MB), 0: shard every weight."""
        check(_lib.load().ort_cuda_set_replicate_bytes(self.handle, int(nbytes)),
              "ort_cuda_set_replicate_bytes")

    def weight_columns(self, name: str) -> Tuple[int, int]:
        """(n0, nl): the columns of `name` this rank holds and computes."""
        n0, nl = ctypes.c_int64(), ctypes.c_int64()
        check(_lib.load().ort_cuda_weight_columns(self.handle, name.encode(), ctypes.byref(n0),
                                                  ctypes.byref(nl)), "ort_cuda_weight_columns")
        return n0.value, nl.value

    def sync(self) -> None:
        check(_lib.load().ort_cuda_sync(self.handle), "ort_cuda_sync")

    def gemv_plan(self, name: str, m: int) -> int:
        """Decode-GEMV plan chosen for weight `name` at M=m (-1: none yet)."""
        p = ctypes.c_int()
        check(_lib.load().ort_cuda_gemv_plan_get(self.handle, name.encode(), m, ctypes.byref(p)),
              "ort_cuda_gemv_plan_get")
        return p.value

    def set_gemv_plan(self, name: str, m: int, plan: int) -> None:
        """Sets (or with -1 clears) the decode-GEMV plan of `name` at M=m."""
        check(_lib.load().ort_cuda_gemv_plan_set(self.handle, name.encode(), m, plan),
              "ort_cuda_gemv_plan_set")

    def launch_count(self) -> int:
        c = ctypes.c_int64()
        check(_lib.load().ort_cuda_launch_count(self.handle, ctypes.byref(c)))
        return c.value

    # -- per-op-type device profile (ExecutionProfile, onnx_graph.dart:22-47) --
    def profile(self, on: bool = True) -> None:
        """Starts (or stops) recording device time per op type."""
        check(_lib.load().ort_cuda_profile_enable(self.handle, int(on)),
              "ort_cuda_profile_enable")

    def profile_reset(self) -> None:
        check(_lib.load().ort_cuda_profile_reset(self.handle), "ort_cuda_profile_reset")

    def profile_entries(self) -> List[tuple]:
        """[(op type, calls, device microseconds)], longest first."""
        L = _lib.load()
        out, i = [], 0
        buf = ctypes.create_string_buffer(64)
        calls, us = ctypes.c_int64(), ctypes.c_double()
        while True:
            rc = L.ort_cuda_profile_read(self.handle, i, buf, 64, ctypes.byref(calls),
                                         ctypes.byref(us))
            if rc == _lib.ERR_NOT_FOUND:
                return out
            check(rc, "ort_cuda_profile_read")
            out.append((buf.value.decode(), calls.value, us.value))
            i += 1

    def profile_report(self) -> str:
        """The text of ExecutionProfile.report(): `op  calls  ms  share%`,
        sorted by cumulative time, then the total."""
        ent = self.profile_entries()
        total = sum(us for _, _, us in ent)
        lines = [f"{'op':<22}{'calls':>7}{'ms':>10}{'share':>8}"]
        for op, n, us in ent:
            share = f"{us * 100 / total:.1f}%" if total else ""
            lines.append(f"{op:<22}{n:>7}{us / 1000:>10.1f}{share:>8}")
        lines.append(f"{'total':<29}{total / 1000:>10.1f}")
        return "\n".join(lines)

    def probe_ffma_tflops(self) -> float:
        """Measured fp32 FFMA throughput of this session's GPU (TFLOP/s)."""
        v = ctypes.c_double()
        check(_lib.load().ort_cuda_probe_ffma(self.handle, ctypes.byref(v)),
              "ort_cuda_probe_ffma")
        return v.value

    # -- CUDA graphs of device-pointer call sequences -----------------------
    def graph_begin(self) -> None:
        """Records the following device-pointer calls instead of running
        them (run each once before, so no buffer grows during capture)."""
        check(_lib.load().ort_cuda_graph_begin(self.handle), "ort_cuda_graph_begin")

    def graph_end(self) -> int:
        gid = ctypes.c_int()
        check(_lib.load().ort_cuda_graph_end(self.handle, ctypes.byref(gid)), "ort_cuda_graph_end")
        return gid.value

    def graph_launch(self, graph_id: int) -> None:
        check(_lib.load().ort_cuda_graph_launch(self.handle, graph_id), "ort_cuda_graph_launch")

    def graph_drop(self, graph_id: int) -> None:
        check(_lib.load().ort_cuda_graph_drop(self.handle, graph_id), "ort_cuda_graph_drop")

    # -- weight residency (uploaded once per session) ----------------------
    def upload_nbits(self, name: str, b_q: np.ndarray, scales: np.ndarray,
                     zero_points: Optional[np.ndarray], *, k: int, n: int, bits: int = 4,
                     block_size: int, zp_per_column: bool = False) -> None:
        b_q = np.ascontiguousarray(b_q, dtype=np.uint8)
        flags = _lib.ZP_PER_COLUMN if zp_per_column else _lib.ZP_FLAT
        if scales.dtype == np.float16:
            sc = np.ascontiguousarray(scales).view(np.uint16)
            flags |= _lib.SCALES_F16
        else:
            sc = np.ascontiguousarray(scales, dtype=np.float32)
        zp = None if zero_points is None else np.ascontiguousarray(zero_points, dtype=np.uint8)
        if bits == 4:
            nb = (k + block_size - 1) // block_size if block_size > 0 else 0
            if b_q.size < n * nb * (block_size // 2):
                raise ValueError(f"MatMulNBits: B has {b_q.size} bytes, expected "
                                 f"{n * nb * (block_size // 2)}")
            if sc.size < n * nb:
                raise ValueError(f"MatMulNBits: scales has {sc.size} values, expected {n * nb}")
            if zp is not None:
                need = (n * ((nb + 1) // 2)) if zp_per_column else (n * nb + 1) // 2
                if zp.size < need:
                    raise ValueError(f"MatMulNBits: zero_points has {zp.size} bytes, "
                                     f"expected {need}")
        check(_lib.load().ort_cuda_upload_nbits(self.handle, name.encode(), b_q.ctypes.data,
                                                sc.ctypes.data, _ptr(zp), k, n, bits,
                                                block_size, flags), "ort_cuda_upload_nbits")
        self.weights[name] = ("nbits", k, n)

    def upload_nbits_file(self, name: str, path: str, *, b_offset: int, scales_offset: int,
                          zp_offset: Optional[int], k: int, n: int, block_size: int,
                          bits: int = 4, scales_f16: bool = False,
                          zp_per_column: bool = False) -> None:
        """A MatMulNBits weight read straight from an external-data file
        (ort_cuda_upload_nbits_file): byte offsets of B, scales and zero
        points (None: no zero points) in `path`."""
        flags = (_lib.ZP_PER_COLUMN if zp_per_column else _lib.ZP_FLAT) | \
            (_lib.SCALES_F16 if scales_f16 else 0)
        check(_lib.load().ort_cuda_upload_nbits_file(
            self.handle, name.encode(), os.fsencode(path), b_offset, scales_offset,
            -1 if zp_offset is None else zp_offset, k, n, bits, block_size, flags),
            "ort_cuda_upload_nbits_file")
        self.weights[name] = ("nbits", k, n)

    def upload_int8(self, name: str, b: np.ndarray, b_zp=None) -> None:
        """MatMulInteger weight B [K, N] (int8 or uint8) with optional zero
        points (scalar or per column, B's type)."""
        b = np.ascontiguousarray(b)
        if b.dtype not in (np.int8, np.uint8) or b.ndim != 2:
            raise ValueError("MatMulInteger: B must be a 2-D int8 or uint8 array")
        zp = None if b_zp is None else np.ascontiguousarray(b_zp, dtype=b.dtype).reshape(-1)
        k, n = b.shape
        check(_lib.load().ort_cuda_upload_int8(self.handle, name.encode(), b.ctypes.data, k, n,
                                               int(b.dtype == np.int8), _ptr(zp),
                                               0 if zp is None else zp.size),
              "ort_cuda_upload_int8")
        self.weights[name] = ("int8", k, n)

    def matmul_integer(self, name: str, a, a_zp=None):
        """Y = (A - a_zp) . (B - b_zp) as int32 (opMatMulInteger).  A numpy
        array (host, synchronous) gives numpy; a torch CUDA tensor (with a_zp
        a torch CUDA tensor or None) gives a torch int32 tensor."""
        kind, k, n = self.weights[name]
        if kind != "int8":
            raise ValueError(f"weight '{name}' is not a MatMulInteger weight")
        shape = tuple(a.shape)
        if shape[-1] != k:
            raise ValueError(f"MatMulInteger: A last dim {shape[-1]} != K {k}")
        m = int(np.prod(shape[:-1], dtype=np.int64)) if len(shape) > 1 else 1
        L = _lib.load()
        if hasattr(a, "data_ptr"):
            import torch
            self._follow_torch_stream()
            signed = a.dtype == torch.int8
            a = a.contiguous()
            zp = None if a_zp is None else a_zp.reshape(-1).contiguous()
            y = torch.empty(shape[:-1] + (n,), dtype=torch.int32, device=a.device)
            check(L.ort_cuda_matmul_integer(self.handle, name.encode(), a.data_ptr(), m,
                                            int(signed), 0 if zp is None else zp.data_ptr(),
                                            0 if zp is None else zp.numel(), y.data_ptr(), 0),
                  "ort_cuda_matmul_integer")
            return y
        a = np.ascontiguousarray(a)
        if a.dtype not in (np.int8, np.uint8):
            raise ValueError("MatMulInteger: A must be int8 or uint8")
        zp = None if a_zp is None else np.ascontiguousarray(a_zp, dtype=a.dtype).reshape(-1)
        y = np.empty(shape[:-1] + (n,), np.int32)
        check(L.ort_cuda_matmul_integer(self.handle, name.encode(), a.ctypes.data, m,
                                        int(a.dtype == np.int8), _ptr(zp),
                                        0 if zp is None else zp.size, y.ctypes.data,
                                        _lib.HOST_IO), "ort_cuda_matmul_integer")
        return y

    def dynamic_quantize_linear(self, x):
        """(y uint8, scale fp32, zero point uint8) of opDynamicQuantizeLinear.
        A torch CUDA tensor gives torch tensors on its device (stream-ordered);
        a numpy array gives (numpy uint8 array, float, int)."""
        L = _lib.load()
        if hasattr(x, "data_ptr"):
            import torch
            self._follow_torch_stream()
            x = x.contiguous().float()
            y = torch.empty(x.shape, dtype=torch.uint8, device=x.device)
            sc = torch.empty((), dtype=torch.float32, device=x.device)
            zp = torch.empty((), dtype=torch.uint8, device=x.device)
            check(L.ort_cuda_dynamic_quantize_linear(self.handle, x.data_ptr(), x.numel(),
                                                     y.data_ptr(), sc.data_ptr(), zp.data_ptr(),
                                                     0), "ort_cuda_dynamic_quantize_linear")
            return y, sc, zp
        a = np.ascontiguousarray(x, dtype=np.float32)
        y = np.empty(a.shape, np.uint8)
        sc = np.zeros(1, np.float32)
        zp = np.zeros(1, np.uint8)
        check(L.ort_cuda_dynamic_quantize_linear(self.handle, a.ctypes.data, a.size, y.ctypes.data,
                                                 sc.ctypes.data, zp.ctypes.data, _lib.HOST_IO),
              "ort_cuda_dynamic_quantize_linear")
        return y, float(sc[0]), int(zp[0])

    def upload_dense(self, name: str, b: np.ndarray, trans_b: bool = False) -> None:
        b = np.ascontiguousarray(b, dtype=np.float32)
        if b.ndim != 2:
            raise ValueError("dense weight must be rank 2")
        check(_lib.load().ort_cuda_upload_dense(self.handle, name.encode(), b.ctypes.data,
                                                b.shape[0], b.shape[1], int(trans_b)),
              "ort_cuda_upload_dense")
        k, n = (b.shape[1], b.shape[0]) if trans_b else b.shape
        self.weights[name] = ("dense", k, n)

    def drop_weight(self, name: str) -> None:
        check(_lib.load().ort_cuda_drop_weight(self.handle, name.encode()), "drop_weight")
        self.weights.pop(name, None)

    # -- ops -----------------------------------------------------------------
    def _run(self, fn, name, a: Tensorish, m: int, k: int, n: int, out_shape, extra=(),
             flags: int = 0, out: Optional[DeviceTensor] = None):
        L = _lib.load()
        if isinstance(a, DeviceTensor):
            y = out if out is not None else DeviceTensor(self, out_shape)
            check(fn(self.handle, name.encode(), a.ptr, m, *extra, y.ptr, flags), fn.__name__)
            return y
        if hasattr(a, "data_ptr"):  # torch CUDA tensor: device pointers
            self._follow_torch_stream()
            y = out
            if y is None:
                import torch
                y = torch.empty(out_shape, dtype=torch.float32, device=a.device)
            check(fn(self.handle, name.encode(), a.data_ptr(), m, *extra, _ptr(y), flags),
                  fn.__name__)
            return y
        a = np.ascontiguousarray(a, dtype=np.float32)
        if out is not None:
            if (not isinstance(out, np.ndarray) or out.dtype != np.float32
                    or not out.flags.c_contiguous or out.size != int(np.prod(out_shape))):
                raise ValueError("out must be a contiguous float32 array of the output size")
            y = out
        else:
            y = np.empty(out_shape, np.float32)
        check(fn(self.handle, name.encode(), a.ctypes.data, m, *extra, y.ctypes.data,
                 flags | _lib.HOST_IO), fn.__name__)
        del L
        return y

    def argmax(self, x, *, is_min: bool = False, select_last: bool = False,
               keepdims: bool = False):
        """ArgMax (ArgMin) over the last axis with the reference's tie and
        NaN rules (opArgMinMax, lib/src/onnx_ops.dart:2198-2237).  A torch
        CUDA tensor gives a torch int64 tensor on its device (stream-ordered);
        a numpy array or a DeviceTensor gives a numpy int64 array."""
        L = _lib.load()
        shape = tuple(x.shape)
        if not shape or shape[-1] < 1:
            raise ValueError("ArgMax needs a non-empty last axis")
        cols = shape[-1]
        rows = int(np.prod(shape[:-1], dtype=np.int64)) if len(shape) > 1 else 1
        out_shape = shape[:-1] + ((1,) if keepdims else ())
        flags = (_lib.ARG_MIN if is_min else 0) | (_lib.ARG_SELECT_LAST if select_last else 0)
        if hasattr(x, "data_ptr"):  # torch CUDA tensor
            import torch
            self._follow_torch_stream()
            x = x.contiguous().float()
            out = torch.empty(out_shape, dtype=torch.int64, device=x.device)
            check(L.ort_cuda_argmax(self.handle, x.data_ptr(), rows, cols, cols, out.data_ptr(),
                                    flags), "ort_cuda_argmax")
            return out
        if isinstance(x, DeviceTensor):
            p = ctypes.c_void_p()
            check(L.ort_cuda_alloc(self.handle, rows * 8, ctypes.byref(p)), "ort_cuda_alloc")
            try:
                check(L.ort_cuda_argmax(self.handle, x.ptr, rows, cols, cols, p.value, flags),
                      "ort_cuda_argmax")
                out = np.empty(out_shape, np.int64)
                check(L.ort_cuda_d2h(self.handle, out.ctypes.data, p.value, rows * 8),
                      "ort_cuda_d2h")
            finally:
                check(L.ort_cuda_free(self.handle, p.value), "ort_cuda_free")
            return out
        a = np.ascontiguousarray(x, dtype=np.float32)
        out = np.empty(out_shape, np.int64)
        check(L.ort_cuda_argmax(self.handle, a.ctypes.data, rows, cols, cols, out.ctypes.data,
                                flags | _lib.HOST_IO), "ort_cuda_argmax")
        return out

    def topk(self, x, k: int, *, largest: bool = True):
        """TopK over the last axis (opTopK, lib/src/onnx_ops.dart:2261-2303):
        (values, int64 indices) of shape x.shape[:-1] + (k,), the
        reference's ordering.  A torch CUDA tensor stays on its device
        (stream-ordered); a numpy array runs through host buffers."""
        L = _lib.load()
        shape = tuple(int(d) for d in x.shape)
        cols = shape[-1] if shape else 1
        rows = int(np.prod(shape[:-1], dtype=np.int64)) if len(shape) > 1 else 1
        flags = 0 if largest else _lib.TOPK_SMALLEST
        out_shape = shape[:-1] + (k,)
        if hasattr(x, "data_ptr"):
            import torch
            self._follow_torch_stream()
            x = x.contiguous().float()
            v = torch.empty(out_shape, dtype=torch.float32, device=x.device)
            i = torch.empty(out_shape, dtype=torch.int64, device=x.device)
            check(L.ort_cuda_topk(self.handle, x.data_ptr(), rows, cols, cols, k, v.data_ptr(),
                                  i.data_ptr(), flags), "ort_cuda_topk")
            return v, i
        a = np.ascontiguousarray(x, dtype=np.float32)
        v = np.empty(out_shape, np.float32)
        i = np.empty(out_shape, np.int64)
        check(L.ort_cuda_topk(self.handle, a.ctypes.data, rows, cols, cols, k, v.ctypes.data,
                              i.ctypes.data, flags | _lib.HOST_IO), "ort_cuda_topk")
        return v, i

    def slice_last_seq(self, x):
        """_SliceLastSeq (onnx_graph.dart:456-473) of a torch CUDA tensor
        [..., seq, inner]: the last position, [..., 1, inner], on the device."""
        import torch
        self._follow_torch_stream()
        x = x.contiguous().float()
        seq, inner = int(x.shape[-2]), int(x.shape[-1])
        if seq <= 1:
            return x
        outer = int(np.prod(x.shape[:-2], dtype=np.int64)) if x.dim() > 2 else 1
        y = torch.empty(tuple(x.shape[:-2]) + (1, inner), dtype=torch.float32, device=x.device)
        check(_lib.load().ort_cuda_slice_last_seq(self.handle, x.data_ptr(), outer, seq, inner,
                                                  y.data_ptr(), 0), "ort_cuda_slice_last_seq")
        return y

    # -- attention of a decoder step ---------------------------------------
    @staticmethod
    def _is_torch(x) -> bool:
        return hasattr(x, "data_ptr")

    def _vals(self, xs):
        """(pointers, host flag) for a call whose tensors are all numpy
        arrays (ORT_CUDA_HOST_IO) or all torch CUDA tensors (device)."""
        present = [x for x in xs if x is not None]
        dev = [self._is_torch(x) for x in present]
        if any(dev) and not all(dev):
            raise ValueError("attention: mix of host and device tensors")
        if dev and all(dev):
            import torch
            self._follow_torch_stream()
            ts = [None if x is None else x.contiguous().to(torch.float32) if x.dtype.is_floating_point
                  else x.contiguous() for x in xs]
            return ts, [0 if t is None else t.data_ptr() for t in ts], 0
        arrs = [None if x is None else np.ascontiguousarray(x) for x in xs]
        arrs = [a if a is None or a.dtype == np.int64 else a.astype(np.float32, copy=False)
                for a in arrs]
        return arrs, [0 if a is None else a.ctypes.data for a in arrs], _lib.HOST_IO

    def group_query_attention(self, q, k, v, num_heads: int, kv_num_heads: int, scale=None,
                              do_rotary: bool = False, rotary_interleaved: bool = False,
                              cos_cache=None, sin_cache=None, past_key=None, past_value=None,
                              attention_bias=None, *, past_len: Optional[int] = None,
                              present_key=None, present_value=None):
        """GroupQueryAttention (opGroupQueryAttention, lib/src/onnx_ops.dart:
        1507-1650) -> (out, present_key, present_value).  numpy inputs run
        through host buffers; torch CUDA tensors stay on the device.  With
        device ``present_key/present_value`` of shape [batch, kv_heads,
        capacity, head] (an in-place KV cache: they may be past_key /
        past_value themselves) ``past_len`` rows are taken as the past and
        this step's rows are appended at past_len."""
        L = _lib.load()
        batch, seq = int(q.shape[0]), int(q.shape[1])
        D = int(q.shape[2]) // num_heads
        cap = 0
        if present_key is not None:
            if not self._is_torch(present_key) or past_len is None:
                raise ValueError("an in-place KV cache needs device tensors and past_len")
            cap = int(present_key.shape[2])
        if past_len is None:
            past_len = int(past_key.shape[2]) if past_key is not None and past_key.ndim == 4 else 0
        T = past_len + seq
        if not past_len:
            past_key = past_value = None
        flags = (_lib.ROTARY if do_rotary else 0) | (_lib.ROTARY_INTERLEAVED if rotary_interleaved else 0)
        ts, ptrs, hflag = self._vals([q, k, v, past_key, past_value,
                                      cos_cache if do_rotary else None,
                                      sin_cache if do_rotary else None, attention_bias])
        cos_t = ts[5]
        max_pos = int(cos_t.shape[0]) if do_rotary else 0
        half = int(cos_t.shape[-1]) if do_rotary else 0
        bias_t = ts[7]
        bb, bh = (int(bias_t.shape[0]), int(bias_t.shape[1])) if bias_t is not None else (0, 0)
        if hflag:
            out = np.empty((batch, seq, num_heads * D), np.float32)
            pk = np.empty((batch, kv_num_heads, T, D), np.float32)
            pv = np.empty_like(pk)
            outp, pkp, pvp = out.ctypes.data, pk.ctypes.data, pv.ctypes.data
        else:
            import torch
            out = torch.empty((batch, seq, num_heads * D), dtype=torch.float32, device=q.device)
            if present_key is None:
                pk = torch.empty((batch, kv_num_heads, T, D), dtype=torch.float32, device=q.device)
                pv = torch.empty_like(pk)
            else:
                pk, pv = present_key, present_value
            outp, pkp, pvp = out.data_ptr(), pk.data_ptr(), pv.data_ptr()
        check(L.ort_cuda_group_query_attention(
            self.handle, ptrs[0], ptrs[1], ptrs[2], ptrs[3], ptrs[4], batch, seq, past_len,
            num_heads, kv_num_heads, D, 0.0 if scale is None else float(scale), ptrs[5],
            ptrs[6], half, max_pos, ptrs[7], bb, bh, cap, outp, pkp, pvp, flags | hflag),
            "ort_cuda_group_query_attention")
        return out, pk, pv

    def multi_head_attention(self, q, k, v, num_heads: int, scale=None, attention_bias=None):
        """MultiHeadAttention (opMultiHeadAttention, lib/src/onnx_ops.dart:
        1656-1725) over already-projected [batch, seq, hidden] Q/K/V."""
        L = _lib.load()
        batch, seq, hidden = (int(d) for d in q.shape)
        kv_seq = int(k.shape[1])
        ts, ptrs, hflag = self._vals([q, k, v, attention_bias])
        bias_t = ts[3]
        bb, bh = (int(bias_t.shape[0]), int(bias_t.shape[1])) if bias_t is not None else (0, 0)
        if hflag:
            out = np.empty((batch, seq, hidden), np.float32)
            outp = out.ctypes.data
        else:
            import torch
            out = torch.empty((batch, seq, hidden), dtype=torch.float32, device=q.device)
            outp = out.data_ptr()
        check(L.ort_cuda_multi_head_attention(
            self.handle, ptrs[0], ptrs[1], ptrs[2], batch, seq, kv_seq, num_heads, hidden,
            0.0 if scale is None else float(scale), ptrs[3], bb, bh, outp, hflag),
            "ort_cuda_multi_head_attention")
        return out

    def fused_sdpa(self, a, b, v, mask, scale: float):
        """_FusedSDPA (opFusedSDPA, lib/src/onnx_ops.dart:1733-1774):
        softmax(a.b * scale + mask) . v for a [..., seq, D], b [..., D,
        kv_seq] (K transposed), v [..., kv_seq, Dv] with equal leading dims
        (at most two); mask broadcasts numpy-style (or None)."""
        L = _lib.load()
        lead = tuple(int(d) for d in a.shape[:-2])
        if len(lead) > 2 or tuple(b.shape[:-2]) != lead or tuple(v.shape[:-2]) != lead:
            raise UnsupportedError("fused SDPA: A, B and V need the same (at most two) batch dims")
        n0, n1 = ((1, 1) + lead)[-2:]
        seq, D = int(a.shape[-2]), int(a.shape[-1])
        kv_seq, Dv = int(b.shape[-1]), int(v.shape[-1])
        ts, ptrs, hflag = self._vals([a, b, v, mask])
        strides = (ctypes.c_int64 * 4)(0, 0, 0, 0)
        if ts[3] is not None:
            m = ts[3]
            mshape = (1,) * (4 - m.ndim) + tuple(int(d) for d in m.shape)
            if m.ndim > 4:
                raise UnsupportedError("fused SDPA: mask of rank > 4")
            full = (n0, n1, seq, kv_seq)
            st, acc = [0, 0, 0, 0], 1
            for i in range(3, -1, -1):
                if mshape[i] not in (1, full[i]):
                    raise ValueError(f"fused SDPA: mask shape {tuple(m.shape)} does not broadcast")
                st[i] = 0 if mshape[i] == 1 else acc
                acc *= mshape[i]
            for i in range(4):
                strides[i] = st[i]
        if hflag:
            out = np.empty(lead + (seq, Dv), np.float32)
            outp = out.ctypes.data
        else:
            import torch
            out = torch.empty(lead + (seq, Dv), dtype=torch.float32, device=a.device)
            outp = out.data_ptr()
        check(L.ort_cuda_fused_sdpa(self.handle, ptrs[0], ptrs[1], ptrs[2], ptrs[3], strides,
                                    n0, n1, seq, kv_seq, D, Dv, float(scale), outp, hflag),
              "ort_cuda_fused_sdpa")
        return out

    def rotary_embedding(self, x, position_ids, cos_cache, sin_cache, interleaved: bool = False,
                         num_heads: int = 0, rotary_dim: int = 0):
        """RotaryEmbedding (opRotaryEmbedding, lib/src/onnx_ops.dart:
        2121-2172); x [batch, seq, hidden] or [batch, heads, seq, head]."""
        L = _lib.load()
        half = int(cos_cache.shape[-1])
        rdim = rotary_dim if rotary_dim > 0 else 2 * half
        if x.ndim == 4:
            batch, heads, seq, head = (int(d) for d in x.shape)
            layout = _lib.ROTARY_BHSD
        else:
            batch, seq, hidden = (int(d) for d in x.shape)
            head = hidden // num_heads if num_heads > 0 else rdim
            heads = hidden // head
            layout = 0
        per_batch = 1 if np.ndim(position_ids) == 2 and int(position_ids.shape[0]) == batch and batch > 1 else 0
        if self._is_torch(x):
            import torch
            position_ids = position_ids.to(torch.int64)
        else:
            position_ids = np.asarray(position_ids).astype(np.int64)
        ts, ptrs, hflag = self._vals([x, position_ids, cos_cache, sin_cache])
        if hflag:
            y = np.empty(tuple(x.shape), np.float32)
            yp = y.ctypes.data
        else:
            import torch
            y = torch.empty(tuple(x.shape), dtype=torch.float32, device=x.device)
            yp = y.data_ptr()
        check(L.ort_cuda_rotary_embedding(
            self.handle, ptrs[0], ptrs[1], per_batch, ptrs[2], ptrs[3], int(ts[2].shape[0]),
            half, batch, seq, heads, head, rotary_dim,
            yp, layout | (_lib.ROTARY_INTERLEAVED if interleaved else 0) | hflag),
            "ort_cuda_rotary_embedding")
        return y

    def fuse_nbits(self, fused: str, names: Sequence[str], drop_parts: bool = False) -> None:
        """One weight `fused` whose columns are those of `names` side by
        side (ort_cuda_fuse_nbits): sibling nodes that read the same input
        (q/k/v, gate/up) then run as one operation (matmul_nbits_group)."""
        parts = [self.weights[n] for n in names]
        k = parts[0][1]
        arr = (ctypes.c_char_p * len(names))(*[n.encode() for n in names])
        check(_lib.load().ort_cuda_fuse_nbits(self.handle, fused.encode(), arr, len(names),
                                              _lib.FUSE_DROP_PARTS if drop_parts else 0),
              "ort_cuda_fuse_nbits")
        widths = [p[2] for p in parts]
        self.weights[fused] = ("nbits", k, sum(widths))
        self._groups = getattr(self, "_groups", {})
        self._groups[fused] = widths
        if drop_parts and self.world == 1:  # a sharded session keeps the parts
            for n in names:
                self.weights.pop(n, None)

    def matmul_nbits_group(self, fused: str, a, flags: int = 0, outs=None):
        """Every part of a fused group on the same A (ort_cuda_matmul_nbits_group):
        a list of outputs, part by part.  A torch CUDA tensor gives torch
        tensors (stream-ordered); a numpy array runs through host buffers."""
        kind, k, _ = self.weights[fused]
        widths = self._groups[fused]
        shape = tuple(a.shape)
        if shape[-1] != k:
            raise ValueError(f"MatMulNBits: A last dim {shape[-1]} != K {k}")
        m = int(np.prod(shape[:-1], dtype=np.int64)) if len(shape) > 1 else 1
        L = _lib.load()
        if hasattr(a, "data_ptr"):
            import torch
            self._follow_torch_stream()
            a = a.contiguous()
            if outs is None:
                outs = [torch.empty(shape[:-1] + (w,), dtype=torch.float32, device=a.device)
                        for w in widths]
            ptrs = (ctypes.c_void_p * len(outs))(*[o.data_ptr() for o in outs])
            check(L.ort_cuda_matmul_nbits_group(self.handle, fused.encode(), a.data_ptr(), m,
                                                ptrs, flags), "ort_cuda_matmul_nbits_group")
            return outs
        a = np.ascontiguousarray(a, dtype=np.float32)
        outs = [np.empty(shape[:-1] + (w,), np.float32) for w in widths]
        ptrs = (ctypes.c_void_p * len(outs))(*[o.ctypes.data for o in outs])
        check(L.ort_cuda_matmul_nbits_group(self.handle, fused.encode(), a.ctypes.data, m, ptrs,
                                            flags | _lib.HOST_IO), "ort_cuda_matmul_nbits_group")
        return outs

    def matmul_nbits_argmax(self, name: str, a, *, is_min: bool = False,
                            select_last: bool = False, logits: bool = False, flags: int = 0):
        """MatMulNBits followed by ArgMax (ArgMin) over the last axis of its
        output, fused on the device (ort_cuda_matmul_nbits_argmax): the
        greedy selection after lm_head.  Returns the int64 indices of shape
        a.shape[:-1] (and the logits when logits=True).  A torch CUDA tensor
        stays on its device (stream-ordered); a numpy array runs through
        host buffers, synchronously."""
        kind, k, n = self.weights[name]
        shape = tuple(a.shape)
        if shape[-1] != k:
            raise ValueError(f"MatMulNBits: A last dim {shape[-1]} != K {k}")
        m = int(np.prod(shape[:-1], dtype=np.int64)) if len(shape) > 1 else 1
        flags |= (_lib.ARG_MIN if is_min else 0) | (_lib.ARG_SELECT_LAST if select_last else 0)
        L = _lib.load()
        if hasattr(a, "data_ptr"):
            import torch
            self._follow_torch_stream()
            a = a.contiguous()
            idx = torch.empty(shape[:-1], dtype=torch.int64, device=a.device)
            y = torch.empty(shape[:-1] + (n,), dtype=torch.float32, device=a.device) \
                if logits else None
            check(L.ort_cuda_matmul_nbits_argmax(self.handle, name.encode(), a.data_ptr(), m,
                                                 idx.data_ptr(), _ptr(y), flags),
                  "ort_cuda_matmul_nbits_argmax")
            return (idx, y) if logits else idx
        a = np.ascontiguousarray(a, dtype=np.float32)
        idx = np.empty(shape[:-1], np.int64)
        y = np.empty(shape[:-1] + (n,), np.float32) if logits else None
        check(L.ort_cuda_matmul_nbits_argmax(self.handle, name.encode(), a.ctypes.data, m,
                                             idx.ctypes.data, _ptr(y), flags | _lib.HOST_IO),
              "ort_cuda_matmul_nbits_argmax")
        return (idx, y) if logits else idx

    def matmul_nbits(self, name: str, a: Tensorish, flags: int = 0, out=None):
        kind, k, n = self.weights[name]
        shape = tuple(a.shape)
        if shape[-1] != k:
            raise ValueError(f"MatMulNBits: A last dim {shape[-1]} != K {k}")
        m = int(np.prod(shape[:-1], dtype=np.int64)) if len(shape) > 1 else 1
        return self._run(_lib.load().ort_cuda_matmul_nbits, name, a, m, k, n,
                         shape[:-1] + (n,), flags=flags, out=out)

    def matmul(self, name: str, a: Tensorish, flags: int = 0, out=None):
        kind, k, n = self.weights[name]
        shape = tuple(a.shape)
        assert len(shape) >= 2 and shape[-1] == k, f"MatMul inner dims mismatch: {shape[-1]} vs {k}"
        m = int(np.prod(shape[:-1], dtype=np.int64))
        return self._run(_lib.load().ort_cuda_matmul, name, a, m, k, n, shape[:-1] + (n,),
                         flags=flags, out=out)

    def gemm(self, name: str, a: Tensorish, c=None, *, alpha: float = 1.0, beta: float = 1.0,
             trans_a: bool = False, flags: int = 0, out=None):
        kind, k, n = self.weights[name]
        if len(a.shape) != 2:
            raise ValueError("Gemm: A must be rank 2")
        m = a.shape[1] if trans_a else a.shape[0]
        ka = a.shape[0] if trans_a else a.shape[1]
        if ka != k:
            raise ValueError(f"Gemm: inner dims mismatch: {ka} vs {k}")
        if c is not None:
            cs = tuple(c.shape)
            c2 = (1,) * (2 - len(cs)) + cs if len(cs) < 2 else cs
            if len(c2) != 2:
                raise ValueError(f"Gemm: C rank {len(cs)} not supported")
            cr, cc = c2
        else:
            cr = cc = 0
        if c is not None and not isinstance(c, DeviceTensor) and not hasattr(c, "data_ptr"):
            c = np.ascontiguousarray(c, dtype=np.float32)
        fl = flags | (_lib.TRANS_A if trans_a else 0)
        return self._run(_lib.load().ort_cuda_gemm, name, a, m, k, n, (m, n),
                         extra=(_ptr(c), cr, cc, float(alpha), float(beta)), flags=fl, out=out)

    def matmul_batched(self, a: np.ndarray, b: np.ndarray, flags: int = 0) -> np.ndarray:
        """Activation x activation MatMul with equal (or absent) batch dims."""
        a = np.ascontiguousarray(a, np.float32)
        b = np.ascontiguousarray(b, np.float32)
        m, k = a.shape[-2:]
        k2, n = b.shape[-2:]
        if k != k2:
            raise ValueError(f"MatMul inner dims mismatch: {k} vs {k2}")
        a_batch, b_batch = a.shape[:-2], b.shape[:-2]
        out_batch = np.broadcast_shapes(a_batch, b_batch)
        count = int(np.prod(out_batch)) if out_batch else 1
        b_count = int(np.prod(b_batch)) if b_batch else 1
        stride = 0 if b_count == 1 else k * n
        ab = np.ascontiguousarray(np.broadcast_to(a, tuple(out_batch) + (m, k)))
        if stride:
            b = np.ascontiguousarray(np.broadcast_to(b, tuple(out_batch) + (k, n)))
        y = np.empty(tuple(out_batch) + (m, n), np.float32)
        check(_lib.load().ort_cuda_matmul_batched(self.handle, ab.ctypes.data, b.ctypes.data,
                                                  count, m, k, n, stride, y.ctypes.data,
                                                  flags | _lib.HOST_IO), "matmul_batched")
        return y

    # -- the _dispatch cases -----------------------------------------------
    def register_initializers(self, nodes: List[dict], initializers: Dict[str, np.ndarray]):
        """Load-time upload of every hot-op weight (the residency hook of the
        OnnxGraphExecutor constructor, onnx_graph.dart:90-97).  ``nodes`` are
        dicts with op_type / inputs / attrs."""
        for node in nodes:
            op, ins, attrs = node["op_type"], node["inputs"], node.get("attrs", {})
            if op == "MatMulNBits":
                if len(ins) > 4:
                    raise UnsupportedError("MatMulNBits: g_idx/bias inputs not supported")
                zp = initializers.get(ins[3]) if len(ins) > 3 and ins[3] else None
                self.upload_nbits(ins[1], initializers[ins[1]], initializers[ins[2]], zp,
                                  k=attrs["K"], n=attrs["N"], bits=attrs.get("bits", 4),
                                  block_size=attrs["block_size"])
            elif op == "Gemm" and ins[1] in initializers:
                self.upload_dense(ins[1], initializers[ins[1]],
                                  trans_b=bool(attrs.get("transB", 0)))
            elif op == "MatMul" and ins[1] in initializers and initializers[ins[1]].ndim == 2:
                self.upload_dense(ins[1], initializers[ins[1]], trans_b=False)

    def dispatch(self, node: dict, values: Dict[str, Tensorish]) -> List[Tensorish]:
        """One node of OnnxGraphExecutor._dispatch for the hot ops."""
        op, ins, attrs = node["op_type"], node["inputs"], node.get("attrs", {})
        a = values[ins[0]]
        if op == "MatMulNBits":
            if len(ins) > 4:
                raise UnsupportedError("MatMulNBits: g_idx/bias inputs not supported")
            if attrs.get("bits", 4) != 4:
                raise UnsupportedError(f"MatMulNBits: only bits=4 supported, got {attrs['bits']}")
            return [self.matmul_nbits(ins[1], a)]
        if op == "Gemm":
            c = values.get(ins[2]) if len(ins) > 2 and ins[2] else None
            return [self.gemm(ins[1], a, c, alpha=attrs.get("alpha", 1.0),
                              beta=attrs.get("beta", 1.0),
                              trans_a=bool(attrs.get("transA", 0)))]
        if op == "MatMul":
            if ins[1] in self.weights:
                return [self.matmul(ins[1], a)]
            return [self.matmul_batched(np.asarray(a), np.asarray(values[ins[1]]))]
        if op == "GroupQueryAttention":  # onnx_graph.dart:978-993
            if attrs.get("softcap", 0) or attrs.get("local_window_size", -1) > 0:
                raise UnsupportedError("GroupQueryAttention: softcap / local_window not supported")
            opt = lambda i: values.get(ins[i]) if len(ins) > i and ins[i] else None  # noqa: E731
            return list(self.group_query_attention(
                a, values[ins[1]], values[ins[2]], attrs["num_heads"], attrs["kv_num_heads"],
                scale=attrs.get("scale"), do_rotary=bool(attrs.get("do_rotary", 0)),
                rotary_interleaved=bool(attrs.get("rotary_interleaved", 0)),
                cos_cache=opt(7), sin_cache=opt(8), past_key=opt(3), past_value=opt(4),
                attention_bias=opt(10)))
        if op == "MultiHeadAttention":  # onnx_graph.dart:994-1000
            bias = values.get(ins[5]) if len(ins) > 5 and ins[5] else None
            return [self.multi_head_attention(a, values[ins[1]], values[ins[2]],
                                              attrs["num_heads"], scale=attrs.get("scale"),
                                              attention_bias=bias)]
        if op == "RotaryEmbedding":  # onnx_graph.dart:1001-1005
            return [self.rotary_embedding(a, values[ins[1]], values[ins[2]], values[ins[3]],
                                          interleaved=bool(attrs.get("interleaved", 0)),
                                          num_heads=attrs.get("num_heads", 0),
                                          rotary_dim=attrs.get("rotary_embedding_dim", 0))]
        if op == "TopK":  # onnx_graph.dart:1514-1517 (last axis)
            k = int(np.asarray(values[ins[1]]).ravel()[0])
            axis = attrs.get("axis", -1)
            if axis not in (-1, np.ndim(a) - 1):
                raise UnsupportedError("TopK: the device path takes the last axis")
            return list(self.topk(a, k, largest=bool(attrs.get("largest", 1))))
        if op == "_FusedSDPA":  # onnx_graph.dart:1029-1033
            return [self.fused_sdpa(a, values[ins[1]], values[ins[2]], values[ins[3]],
                                    attrs["scale"])]
        raise UnsupportedError(f"op {op} is not on the CUDA matmul path")


# ---- pure-function mirrors on a throwaway session ----------------------------
_default: Optional[CudaSession] = None


def default_session() -> CudaSession:
    global _default
    if _default is None:
        _default = CudaSession(0)
    return _default


def op_matmul_nbits(a: np.ndarray, b_q: np.ndarray, scales: np.ndarray,
                    zero_points: Optional[np.ndarray], *, k: int, n: int, bits: int,
                    block_size: int, mode: str = "exact") -> np.ndarray:
    """opMatMulNBits (onnx_qlinear_ops.dart:114-156) on the GPU."""
    if bits != 4:
        raise UnsupportedError(f"MatMulNBits: only bits=4 supported, got {bits}")
    s = default_session()
    s.upload_nbits("__op_matmul_nbits", b_q, scales, zero_points, k=k, n=n, bits=bits,
                   block_size=block_size)
    try:
        return s.matmul_nbits("__op_matmul_nbits", a, flags=_lib.flags_mode(_lib.MODES[mode]))
    finally:
        s.drop_weight("__op_matmul_nbits")


def op_gemm(a: np.ndarray, b: np.ndarray, c: Optional[np.ndarray] = None, *, alpha: float = 1.0,
            beta: float = 1.0, trans_a: bool = False, trans_b: bool = False,
            mode: str = "exact") -> np.ndarray:
    """opGemm (onnx_ops.dart:1777-1793) on the GPU."""
    s = default_session()
    s.upload_dense("__op_gemm", b, trans_b=trans_b)
    try:
        return s.gemm("__op_gemm", a, c, alpha=alpha, beta=beta, trans_a=trans_a,
                      flags=_lib.flags_mode(_lib.MODES[mode]))
    finally:
        s.drop_weight("__op_gemm")


def op_matmul(a: np.ndarray, b: np.ndarray, mode: str = "exact") -> np.ndarray:
    """opMatMul (onnx_ops.dart:1375-1431) on the GPU."""
    s = default_session()
    fl = _lib.flags_mode(_lib.MODES[mode])
    if b.ndim == 2:
        s.upload_dense("__op_matmul", b)
        try:
            return s.matmul("__op_matmul", a, flags=fl)
        finally:
            s.drop_weight("__op_matmul")
    return s.matmul_batched(a, b, flags=fl)


__all__ = ["CudaSession", "DeviceTensor", "UnsupportedError", "StateError", "op_matmul_nbits",
           "op_gemm", "op_matmul", "default_session"]
