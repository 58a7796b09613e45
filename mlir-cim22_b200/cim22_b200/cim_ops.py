"""CIM layers and Host glue over CUDA tensors, calling the C ABI.

PyTorch supplies device memory and the current stream; every computation is a
kernel of libcim22_cuda.so. Tensors must be contiguous CUDA tensors.
"""

from __future__ import annotations

import ctypes

import numpy as np
import torch

from . import abi
from .native import CudaError, check, lib

ACT = {None: 0, "none": 0, "relu": 1, "gelu": 2}


def _ptr(t: torch.Tensor | None):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream(device: torch.device | None = None):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _require(t: torch.Tensor, dtype: torch.dtype, name: str) -> None:
    if not t.is_cuda or t.dtype != dtype or not t.is_contiguous():
        raise TypeError(f"{name} must be a contiguous CUDA {dtype} tensor")


class Workspace:
    """Grow-only scratch buffer shared by the layers of one program."""

    def __init__(self, device: torch.device) -> None:
        self.device = device
        self.buffer = torch.empty(0, dtype=torch.uint8, device=device)

    def get(self, nbytes: int) -> torch.Tensor:
        if self.buffer.numel() < nbytes:
            self.buffer = torch.empty(max(nbytes, 2 * self.buffer.numel()), dtype=torch.uint8,
                                      device=self.device)
        return self.buffer


class StatusWord:
    """Device int32 that kernels OR error bits into."""

    def __init__(self, device: torch.device) -> None:
        self.tensor = torch.zeros(1, dtype=torch.int32, device=device)

    def reset(self) -> None:
        self.tensor.zero_()

    def raise_if_set(self, prefix: str = "") -> None:
        raise_status(int(self.tensor.item()), prefix)


def raise_status(value: int, prefix: str = "") -> None:
    """Raise the reference's error text for a nonzero status word."""
    if value:
        message = lib().cim22_cuda_status_message(value).decode()
        raise RuntimeError(f"{prefix}{message}")


class CimLayer:
    """Resident CIM weights of one Linear/Conv contraction (W[n, k])."""

    def __init__(self, weight: np.ndarray | torch.Tensor, *, kind: str = "bf16",
                 device: int | torch.device = 0, compensation: str = "sign-split") -> None:
        """compensation: the BF16 mode, "sign-split" (default), or the
        reference's diagnostic "legacy" and "none" (no sign split)."""
        dev = torch.device("cuda", device) if isinstance(device, int) else torch.device(device)
        self.device = dev
        index = dev.index if dev.index is not None else torch.cuda.current_device()
        w = weight.detach().cpu().numpy() if isinstance(weight, torch.Tensor) else weight
        w = np.ascontiguousarray(w.reshape(w.shape[0], -1))
        self.n, self.k = w.shape
        self.kind = kind
        err = ctypes.create_string_buffer(512)
        self.compensation = compensation
        if kind == "bf16":
            if compensation not in abi.COMPENSATION:
                raise ValueError("BF16 compensation must be sign-split, legacy or none")
            w = np.ascontiguousarray(w, dtype=np.float32)
            self._handle = lib().cim22_cuda_layer_create_bf16_mode(
                index, w.ctypes.data, self.n, self.k, abi.COMPENSATION[compensation], err,
                len(err))
        elif kind == "int8":
            w = np.ascontiguousarray(w, dtype=np.int8)
            self._handle = lib().cim22_cuda_layer_create_int8(index, w.ctypes.data, self.n,
                                                              self.k, err, len(err))
        else:
            raise ValueError(f"unknown CIM layer kind {kind}")
        if not self._handle:
            raise CudaError(err.value.decode())

    def close(self) -> None:
        if getattr(self, "_handle", None):
            lib().cim22_cuda_layer_destroy(self._handle)
            self._handle = None

    def __del__(self) -> None:  # pragma: no cover
        try:
            self.close()
        except Exception:
            pass

    @property
    def fused_forward(self) -> bool:
        """forward_bf16 runs as one kernel (gather + prealign + contraction)."""
        return bool(lib().cim22_cuda_layer_fused_forward(self._handle))

    @property
    def range_safe(self) -> bool:
        return bool(lib().cim22_cuda_layer_range_safe(self._handle))

    @property
    def bf16_operands(self) -> bool:
        """Whether the weights admit the contraction with BF16 operands."""
        return bool(lib().cim22_cuda_layer_bf16_operands(self._handle))

    def workspace_bytes(self, m: int, branches: int = 4) -> int:
        if self.kind == "bf16":
            return int(lib().cim22_cuda_layer_workspace_bf16(self._handle, m, branches))
        return int(lib().cim22_cuda_layer_workspace_int8(self._handle, m))

    def forward_bf16(self, x: torch.Tensor, out: torch.Tensor, m: int, *,
                     gather: abi.Gather | None = None, bias: torch.Tensor | None = None,
                     activation: str | None = None, branches: int = 4,
                     out_pixels: int = 0, post_scale: torch.Tensor | None = None,
                     post_shift: torch.Tensor | None = None,
                     workspace: Workspace, status: StatusWord) -> torch.Tensor:
        """out is [m, n] rows, or NCHW images [m / out_pixels, n, out_pixels]
        when out_pixels > 0; post_scale/post_shift fold a following per-lane
        affine (inference batch norm) into the epilogue."""
        _require(x, torch.float32, "x")
        _require(out, torch.float32, "out")
        if bias is not None:
            _require(bias, torch.float32, "bias")
        nbytes = self.workspace_bytes(m, branches)
        ws = workspace.get(nbytes)
        rc = lib().cim22_cuda_layer_forward_bf16_ex(
            self._handle, _ptr(x), None if gather is None else ctypes.byref(gather), m,
            out_pixels, _ptr(bias), _ptr(post_scale), _ptr(post_shift), ACT[activation],
            branches, _ptr(out), _ptr(ws), ws.numel(), _ptr(status.tensor), _stream(x.device))
        check(rc, "cim22_cuda_layer_forward_bf16")
        return out

    def prepare_bf16(self, x: torch.Tensor, m: int, *, gather: abi.Gather | None = None,
                     branches: int = 4, workspace: Workspace, status: StatusWord) -> None:
        """First kernel of forward_bf16: gather, split and prealign into the workspace."""
        _require(x, torch.float32, "x")
        ws = workspace.get(self.workspace_bytes(m, branches))
        check(lib().cim22_cuda_layer_prepare_bf16(
            self._handle, _ptr(x), None if gather is None else ctypes.byref(gather), m,
            branches, _ptr(ws), ws.numel(), _ptr(status.tensor), _stream(x.device)),
            "cim22_cuda_layer_prepare_bf16")

    def contract_bf16(self, out: torch.Tensor, m: int, *, bias: torch.Tensor | None = None,
                      activation: str | None = None, branches: int = 4,
                      out_pixels: int = 0, post_scale: torch.Tensor | None = None,
                      post_shift: torch.Tensor | None = None,
                      residual: torch.Tensor | None = None,
                      workspace: Workspace, status: StatusWord) -> None:
        """Second kernel of forward_bf16: crossbar dots, restore, accumulate, merge.
        residual (laid out like out) is added after the per-lane fma and before
        the activation, as a Conv -> BatchNorm -> add -> ReLU block computes it."""
        _require(out, torch.float32, "out")
        if residual is not None:
            _require(residual, torch.float32, "residual")
            if residual.numel() != out.numel():
                raise ValueError("residual must have the output's shape")
        ws = workspace.get(self.workspace_bytes(m, branches))
        check(lib().cim22_cuda_layer_contract_bf16_res(
            self._handle, m, out_pixels, _ptr(bias), _ptr(post_scale), _ptr(post_shift),
            _ptr(residual), ACT[activation], branches, _ptr(out), _ptr(ws), ws.numel(),
            _ptr(status.tensor), _stream(out.device)),
            "cim22_cuda_layer_contract_bf16")

    def linear_bf16(self, x: torch.Tensor, bias=None, activation=None, branches: int = 4,
                    workspace: Workspace | None = None,
                    status: StatusWord | None = None) -> torch.Tensor:
        """y[m, n] for x[m, k] (f32 CUDA)."""
        x = x.contiguous()
        m = x.shape[0]
        out = torch.empty(m, self.n, dtype=torch.float32, device=x.device)
        own_status = status is None
        status = status or StatusWord(x.device)
        self.forward_bf16(x, out, m, bias=bias, activation=activation, branches=branches,
                          workspace=workspace or Workspace(x.device), status=status)
        if own_status:
            status.raise_if_set()
        return out

    def forward_int8(self, x: torch.Tensor, out: torch.Tensor, m: int, *,
                     gather: abi.Gather | None = None, pad_bottom: int = -1,
                     pad_right: int = -1, bias: torch.Tensor | None = None,
                     out_pixels: int = 0, exact_unproven: bool = True,
                     workspace: Workspace, status: StatusWord) -> torch.Tensor:
        """INT8 layer over int8 rows [m, k] or a conv gather of an int8 image
        batch; out is int32 [m, n] rows, or NCHW [m / out_pixels, n,
        out_pixels]. bias is int32 [n] (wrapping add). exact_unproven computes
        weights that fail the i21 range proof exactly, as the compiler's Host
        does; otherwise their tiles are checked (CIM22_STATUS_I21_RANGE)."""
        _require(x, torch.int8, "x")
        _require(out, torch.int32, "out")
        if bias is not None:
            _require(bias, torch.int32, "bias")
        ws = workspace.get(self.workspace_bytes(m))
        rc = lib().cim22_cuda_layer_forward_int8_ex(
            self._handle, _ptr(x), None if gather is None else ctypes.byref(gather), m,
            pad_bottom, pad_right, _ptr(bias), out_pixels, int(exact_unproven), _ptr(out),
            _ptr(ws), ws.numel(), _ptr(status.tensor), _stream(x.device))
        check(rc, "cim22_cuda_layer_forward_int8_ex")
        return out

    def conv2d_int8(self, x: torch.Tensor, kernel: tuple[int, int], stride=(1, 1),
                    pads=(0, 0, 0, 0), bias: torch.Tensor | None = None, *,
                    layout: str = "nchw", exact_unproven: bool = True,
                    workspace: Workspace | None = None,
                    status: StatusWord | None = None) -> torch.Tensor:
        """ConvInteger of an int8 image batch (NCHW, or NHWC with layout="nhwc")
        with this layer's [F, C * KH * KW] weights; pads are ONNX's (top, left,
        bottom, right). Returns int32 NCHW [N, F, OH, OW]."""
        kh, kw = kernel
        sh, sw = (stride, stride) if isinstance(stride, int) else stride
        top, left, bottom, right = pads
        if layout == "nchw":
            n, c, h, w = x.shape
            kind = abi.GATHER_CONV_NCHW
        else:
            n, h, w, c = x.shape
            kind = abi.GATHER_CONV_NHWC
        g = abi.Gather()
        g.kind = kind
        g.batch, g.channels, g.height, g.width = n, c, h, w
        g.kernel_h, g.kernel_w, g.stride_h, g.stride_w = kh, kw, sh, sw
        g.pad_h, g.pad_w = top, left
        g.out_h = (h + top + bottom - kh) // sh + 1
        g.out_w = (w + left + right - kw) // sw + 1
        pixels = g.out_h * g.out_w
        out = torch.empty(n, self.n, g.out_h, g.out_w, dtype=torch.int32, device=x.device)
        own_status = status is None
        status = status or StatusWord(x.device)
        self.forward_int8(x.contiguous(), out, n * pixels, gather=g, pad_bottom=bottom,
                          pad_right=right, bias=bias, out_pixels=pixels,
                          exact_unproven=exact_unproven,
                          workspace=workspace or Workspace(x.device), status=status)
        if own_status:
            status.raise_if_set()
        return out

    def linear_int8(self, x: torch.Tensor, workspace: Workspace | None = None,
                    status: StatusWord | None = None) -> torch.Tensor:
        _require(x, torch.int8, "x")
        m = x.shape[0]
        out = torch.empty(m, self.n, dtype=torch.int32, device=x.device)
        workspace = workspace or Workspace(x.device)
        ws = workspace.get(self.workspace_bytes(m))
        own_status = status is None
        status = status or StatusWord(x.device)
        rc = lib().cim22_cuda_layer_forward_int8(self._handle, _ptr(x), m, _ptr(out), _ptr(ws),
                                                 ws.numel(), _ptr(status.tensor),
                                                 _stream(x.device))
        check(rc, "cim22_cuda_layer_forward_int8")
        if own_status:
            status.raise_if_set()
        return out


def conv_gather(kind: int, n: int, c: int, h: int, w: int, kh: int, kw: int, stride: int,
                pad: int) -> abi.Gather:
    g = abi.Gather()
    g.kind = kind
    g.batch, g.channels, g.height, g.width = n, c, h, w
    g.kernel_h, g.kernel_w = kh, kw
    g.stride_h = g.stride_w = stride
    g.pad_h = g.pad_w = pad
    g.out_h = (h + 2 * pad - kh) // stride + 1
    g.out_w = (w + 2 * pad - kw) // stride + 1
    return g


# ---------------------------------------------------------------------------
# Glue.


def relu(x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    out = torch.empty_like(x) if out is None else out
    check(lib().cim22_cuda_relu(_ptr(x), _ptr(out), x.numel(), _stream(x.device)), "relu")
    return out


def gelu(x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    out = torch.empty_like(x) if out is None else out
    check(lib().cim22_cuda_gelu(_ptr(x), _ptr(out), x.numel(), _stream(x.device)), "gelu")
    return out


def add(a: torch.Tensor, b: torch.Tensor, activation: str | None = None,
        out: torch.Tensor | None = None) -> torch.Tensor:
    out = torch.empty_like(a) if out is None else out
    check(lib().cim22_cuda_add(_ptr(a), _ptr(b), _ptr(out), a.numel(), ACT[activation],
                               _stream(a.device)), "add")
    return out


def maxpool2d_nhwc(x: torch.Tensor, kernel: int, stride: int, pad: int = 0,
                   out: torch.Tensor | None = None) -> torch.Tensor:
    n, h, w, c = x.shape
    oh, ow = (h + 2 * pad - kernel) // stride + 1, (w + 2 * pad - kernel) // stride + 1
    out = torch.empty(n, oh, ow, c, dtype=x.dtype, device=x.device) if out is None else out
    check(lib().cim22_cuda_maxpool2d_nhwc(_ptr(x), _ptr(out), n, h, w, c, kernel, stride, pad,
                                          _stream(x.device)), "maxpool2d")
    return out


def avgpool2d_nhwc(x: torch.Tensor, kernel: int, stride: int,
                   out: torch.Tensor | None = None) -> torch.Tensor:
    n, h, w, c = x.shape
    oh, ow = (h - kernel) // stride + 1, (w - kernel) // stride + 1
    out = torch.empty(n, oh, ow, c, dtype=x.dtype, device=x.device) if out is None else out
    check(lib().cim22_cuda_avgpool2d_nhwc(_ptr(x), _ptr(out), n, h, w, c, kernel, stride,
                                          _stream(x.device)), "avgpool2d")
    return out


def global_avgpool_nhwc(x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    n, h, w, c = x.shape
    out = torch.empty(n, c, dtype=x.dtype, device=x.device) if out is None else out
    check(lib().cim22_cuda_global_avgpool_nhwc(_ptr(x), _ptr(out), n, h, w, c,
                                               _stream(x.device)), "global_avgpool")
    return out


def channel_affine_nhwc(x: torch.Tensor, scale: torch.Tensor, shift: torch.Tensor,
                        activation: str | None = None,
                        out: torch.Tensor | None = None) -> torch.Tensor:
    c = x.shape[-1]
    out = torch.empty_like(x) if out is None else out
    check(lib().cim22_cuda_channel_affine_nhwc(_ptr(x), _ptr(scale), _ptr(shift), _ptr(out),
                                               x.numel() // c, c, ACT[activation],
                                               _stream(x.device)), "channel_affine")
    return out


def maxpool2d_nchw(x: torch.Tensor, kernel: int, stride: int, pad: int = 0,
                   out: torch.Tensor | None = None) -> torch.Tensor:
    n, c, h, w = x.shape
    oh, ow = (h + 2 * pad - kernel) // stride + 1, (w + 2 * pad - kernel) // stride + 1
    out = torch.empty(n, c, oh, ow, dtype=x.dtype, device=x.device) if out is None else out
    check(lib().cim22_cuda_maxpool2d_nchw(_ptr(x), _ptr(out), n, c, h, w, kernel, stride, pad,
                                          _stream(x.device)), "maxpool2d")
    return out


def avgpool2d_nchw(x: torch.Tensor, kernel: int, stride: int,
                   out: torch.Tensor | None = None) -> torch.Tensor:
    n, c, h, w = x.shape
    oh, ow = (h - kernel) // stride + 1, (w - kernel) // stride + 1
    out = torch.empty(n, c, oh, ow, dtype=x.dtype, device=x.device) if out is None else out
    check(lib().cim22_cuda_avgpool2d_nchw(_ptr(x), _ptr(out), n, c, h, w, kernel, stride,
                                          _stream(x.device)), "avgpool2d")
    return out


def global_avgpool_nchw(x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    n, c, h, w = x.shape
    out = torch.empty(n, c, dtype=x.dtype, device=x.device) if out is None else out
    check(lib().cim22_cuda_global_avgpool_nchw(_ptr(x), _ptr(out), n, c, h, w,
                                               _stream(x.device)), "global_avgpool")
    return out


def channel_affine_nchw(x: torch.Tensor, scale: torch.Tensor, shift: torch.Tensor,
                        activation: str | None = None,
                        out: torch.Tensor | None = None) -> torch.Tensor:
    """Per-channel affine over [n, c, ...] (every trailing element of a channel)."""
    n, c = x.shape[0], x.shape[1]
    hw = x.numel() // max(1, n * c)
    out = torch.empty_like(x) if out is None else out
    check(lib().cim22_cuda_channel_affine_nchw(_ptr(x), _ptr(scale), _ptr(shift), _ptr(out),
                                               n, c, hw, ACT[activation], _stream(x.device)),
          "channel_affine")
    return out


def unshard_columns(src: torch.Tensor, total: int,
                    out: torch.Tensor | None = None) -> torch.Tensor:
    """[ranks, rows, cols] blocks (an all-gather's stacking) -> [rows, total]."""
    ranks, rows, cols = src.shape
    out = torch.empty(rows, total, dtype=src.dtype, device=src.device) if out is None else out
    check(lib().cim22_cuda_unshard_columns(_ptr(src), _ptr(out), ranks, rows, cols, total,
                                           _stream(src.device)), "unshard_columns")
    return out


def softmax(x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    cols = x.shape[-1]
    out = torch.empty_like(x) if out is None else out
    check(lib().cim22_cuda_softmax(_ptr(x), _ptr(out), x.numel() // cols, cols,
                                   _stream(x.device)), "softmax")
    return out


def nhwc_to_nchw(x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    n, h, w, c = x.shape
    out = torch.empty(n, c, h, w, dtype=x.dtype, device=x.device) if out is None else out
    check(lib().cim22_cuda_nhwc_to_nchw(_ptr(x), _ptr(out), n, h, w, c, _stream(x.device)),
          "nhwc_to_nchw")
    return out


def nchw_to_nhwc(x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    n, c, h, w = x.shape
    out = torch.empty(n, h, w, c, dtype=x.dtype, device=x.device) if out is None else out
    check(lib().cim22_cuda_nchw_to_nhwc(_ptr(x), _ptr(out), n, c, h, w, _stream(x.device)),
          "nchw_to_nhwc")
    return out
