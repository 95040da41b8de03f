"""Functional entry points over libb200fo.so for torch CUDA tensors.

These are the calls the reference-shaped modules (`icpp_tuning_b200.gemm.*`,
`icpp_tuning_b200.conv.*`) are built on.  PyTorch supplies device memory and the current
stream; every FLOP runs in the library's sm_100a kernels.  Tensors must live on a CUDA
device: there is no CPU path, and a missing library raises.
"""
from __future__ import annotations

import ctypes
from typing import Optional

import torch

from . import _native as N

_DT = {torch.float16: N.FO_DT_F16, torch.bfloat16: N.FO_DT_BF16, torch.float32: N.FO_DT_F32}
EPILOGUES = {
    "none": N.FO_EPI_NONE, "bias": N.FO_EPI_BIAS, "bias_relu": N.FO_EPI_BIAS_RELU,
    "bias_gelu_tanh": N.FO_EPI_BIAS_GELU_TANH, "bias_gelu_erf": N.FO_EPI_BIAS_GELU_ERF,
    "bias_layernorm": N.FO_EPI_BIAS_LN, "relu": N.FO_EPI_RELU,
    "bias_residual_layernorm": N.FO_EPI_BIAS_RESIDUAL_LN,
}


def dtype_code(dt: torch.dtype) -> int:
    try:
        return _DT[dt]
    except KeyError:
        raise ValueError(f"unsupported dtype {dt}; use float16, bfloat16 or float32") from None


def _require_cuda(*ts: Optional[torch.Tensor]) -> torch.device:
    dev = None
    for t in ts:
        if t is None:
            continue
        if not t.is_cuda:
            raise ValueError("b200fo operators take CUDA tensors only; there is no CPU path")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise ValueError(f"tensors on different devices: {dev} and {t.device}")
    return dev


def _rows(t: torch.Tensor, name: str) -> int:
    if t.dim() != 2 or t.stride(1) != 1:
        raise ValueError(f"{name} must be a 2-D tensor with unit column stride")
    return t.stride(0)


def _vec(t: Optional[torch.Tensor], n: int, name: str) -> Optional[torch.Tensor]:
    if t is None:
        return None
    if t.dim() != 1 or t.numel() != n or not t.is_contiguous():
        raise ValueError(f"{name} must be a contiguous vector of length {n}")
    return t


def _stream(dev: torch.device, stream) -> int:
    s = torch.cuda.current_stream(dev) if stream is None else stream
    return s.cuda_stream


def default_config(M: int, n: int, K: int, epilogue: str = "none") -> N.FoTileCfg:
    """A reasonable tile when the caller does not pass one (the autotuner picks better)."""
    bn = 256 if n > 128 else (128 if n > 64 else 64)
    stages = {256: 4, 128: 6, 64: 8}[bn]
    return N.tile_cfg(block_n=bn, stages=stages, group_m=0 if epilogue == "bias_layernorm" else 8)


def as_tile_cfg(cfg) -> N.FoTileCfg:
    """Accepts an FoTileCfg or a raw config dict of the autotuner
    (block_M / block_N / block_K / num_stages / group_m / max_ctas / swap_ab / split_k /
    split_mode / ln_mode)."""
    if isinstance(cfg, N.FoTileCfg):
        return cfg
    return N.tile_cfg(block_n=int(cfg["block_N"]), stages=int(cfg["num_stages"]),
                      group_m=int(cfg.get("group_m", 0)), max_ctas=int(cfg.get("max_ctas", 0)),
                      block_m=int(cfg.get("block_M", 128)), block_k=int(cfg.get("block_K", 64)),
                      swap_ab=int(cfg.get("swap_ab", 0)), split_k=int(cfg.get("split_k", 0)),
                      split_mode=int(cfg.get("split_mode", 0)), ln_mode=int(cfg.get("ln_mode", 0)))


class StreamWorkspaces:
    """Zero-filled workspaces of one built operator, one per CUDA stream it runs on.

    The split-K tail and the one-kernel LayerNorm keep counters in their workspace that
    each call leaves zeroed; two calls that overlap on the GPU (on different streams)
    must not share one.  The workspace of the stream current at build time is allocated
    up front; another stream gets its own on its first call (calls on one stream are
    ordered, so they share it)."""

    def __init__(self, nbytes: int, device: Optional[torch.device] = None):
        self.nbytes = int(nbytes)
        self.device = device if device is not None else torch.device("cuda", torch.cuda.current_device())
        self._by_stream = {}
        self.default = self.get(torch.cuda.current_stream(self.device))

    def get(self, stream=None) -> Optional[torch.Tensor]:
        if self.nbytes <= 0:
            return None
        s = torch.cuda.current_stream(self.device) if stream is None else stream
        ws = self._by_stream.get(s.cuda_stream)
        if ws is None:
            with torch.cuda.stream(s):
                ws = torch.zeros(max(16, self.nbytes), dtype=torch.uint8, device=self.device)
            self._by_stream[s.cuda_stream] = ws
        return ws


def workspace_bytes(M: int, N_: int, K: int, epilogue: str, cfg) -> int:
    """Workspace fo_gemm uses for this problem: LayerNorm statistics (required) or, for
    the other epilogues, fp32 partials of the split-K tail (optional, zero-filled)."""
    d = N.FoGemmDesc()
    d.M, d.N, d.K, d.epilogue = M, N_, K, EPILOGUES[epilogue]
    c = as_tile_cfg(cfg)
    return int(N.lib().fo_gemm_workspace_size(ctypes.byref(d), ctypes.byref(c)))


def ln_workspace_bytes(M: int, N_: int, cfg) -> int:
    return workspace_bytes(M, N_, 0, "bias_layernorm", cfg)


def gemm(a: torch.Tensor, b: torch.Tensor, *, b_layout: str = "kn", epilogue: str = "none",
         bias: Optional[torch.Tensor] = None, gamma: Optional[torch.Tensor] = None,
         beta: Optional[torch.Tensor] = None, eps: float = 1e-5,
         out: Optional[torch.Tensor] = None, out_dtype: Optional[torch.dtype] = None,
         workspace: Optional[torch.Tensor] = None, residual: Optional[torch.Tensor] = None,
         config=None, stream=None) -> torch.Tensor:
    """out = epilogue(a @ B) with fp32 accumulation.

    a: [M, K]; b: [K, N] when b_layout == "kn" (reference layout), [N, K] when "nk".
    epilogue: one of EPILOGUES.  "bias_layernorm" needs gamma, beta and a workspace of
    ln_workspace_bytes(M, N, config) bytes for the per-row slice statistics.  The other
    epilogues accept an optional zero-filled workspace of workspace_bytes(...) bytes that
    lets the kernel split the tiles of a partial last wave along K.
    "bias_residual_layernorm" computes LN(a @ B + bias + residual) with the GEMM result
    rounded to the output dtype before the residual add (the fp16 model-layer semantics).
    """
    dev = _require_cuda(a, b, bias, gamma, beta, out, workspace, residual)
    if b_layout not in ("kn", "nk"):
        raise ValueError("b_layout must be 'kn' or 'nk'")
    if a.dtype != b.dtype or a.dtype not in (torch.float16, torch.bfloat16):
        raise ValueError("a and b must share dtype float16 or bfloat16")
    M, K = a.shape
    Nn = b.shape[1] if b_layout == "kn" else b.shape[0]
    Kb = b.shape[0] if b_layout == "kn" else b.shape[1]
    if Kb != K:
        raise ValueError(f"inner dimensions differ: a is [{M},{K}], b gives K={Kb}")
    epi = EPILOGUES[epilogue]
    if out is None:
        out = torch.empty((M, Nn), device=dev, dtype=out_dtype or a.dtype)
    if tuple(out.shape) != (M, Nn):
        raise ValueError(f"out must be [{M},{Nn}]")
    cfg = as_tile_cfg(config) if config is not None else default_config(M, Nn, K, epilogue)
    d = N.FoGemmDesc()
    d.M, d.N, d.K = M, Nn, K
    d.a, d.b, d.out = a.data_ptr(), b.data_ptr(), out.data_ptr()
    d.lda, d.ldb, d.ldo = _rows(a, "a"), _rows(b, "b"), _rows(out, "out")
    d.in_dtype, d.out_dtype = dtype_code(a.dtype), dtype_code(out.dtype)
    d.b_layout = N.FO_B_KN if b_layout == "kn" else N.FO_B_NK
    d.epilogue = epi
    vecs = [_vec(bias, Nn, "bias"), _vec(gamma, Nn, "gamma"), _vec(beta, Nn, "beta")]
    vdt = {v.dtype for v in vecs if v is not None}
    if len(vdt) > 1:
        raise ValueError("bias, gamma and beta must share one dtype")
    d.vec_dtype = dtype_code(vdt.pop()) if vdt else N.FO_DT_F32
    d.bias = bias.data_ptr() if bias is not None else None
    d.gamma = gamma.data_ptr() if gamma is not None else None
    d.beta = beta.data_ptr() if beta is not None else None
    d.eps = float(eps)
    if workspace is not None:
        d.workspace, d.workspace_bytes = workspace.data_ptr(), workspace.numel() * workspace.element_size()
    if residual is not None:
        if tuple(residual.shape) != (M, Nn) or residual.dtype != out.dtype:
            raise ValueError(f"residual must be [{M},{Nn}] of the output dtype")
        d.residual, d.ldr = residual.data_ptr(), _rows(residual, "residual")
    with torch.cuda.device(dev):
        N.check(N.lib().fo_gemm(ctypes.byref(d), ctypes.byref(cfg), _stream(dev, stream)))
    return out


def _conv_desc(n, h, wd, c, f, kh, kw, stride, padding, dilation, out_dtype=N.FO_DT_BF16) -> N.FoConvDesc:
    d = N.FoConvDesc()
    d.n, d.h, d.w, d.c, d.f, d.kh, d.kw = n, h, wd, c, f, kh, kw
    d.stride, d.pad, d.dil = stride, padding, dilation
    d.in_dtype = d.out_dtype = out_dtype
    return d


def conv_workspace_bytes(n, h, w, c, f, kh, kw, stride=1, padding=1, dilation=1, config=None) -> int:
    """Optional zero-filled workspace that lets fo_conv2d split a partial last wave along K."""
    cfg = as_tile_cfg(config) if config is not None else default_conv_config(f)
    d = _conv_desc(n, h, w, c, f, kh, kw, stride, padding, dilation)
    return int(N.lib().fo_conv2d_workspace_size(ctypes.byref(d), ctypes.byref(cfg)))


def default_conv_config(f: int) -> N.FoTileCfg:
    """Operand-swapped 128-channel x 256-pixel tiles (the measured best for few channels)."""
    return N.tile_cfg(block_n=256, stages=4, group_m=0, swap_ab=1)


def conv2d_nhwc(x: torch.Tensor, w: torch.Tensor, *, bias: Optional[torch.Tensor] = None,
                relu: bool = False, stride: int = 1, padding: int = 1, dilation: int = 1,
                out: Optional[torch.Tensor] = None, out_dtype: Optional[torch.dtype] = None,
                workspace: Optional[torch.Tensor] = None, config=None, stream=None,
                bn: Optional[tuple] = None, bn_eps: float = 1e-5,
                residual: Optional[torch.Tensor] = None) -> torch.Tensor:
    """out[n,oh,ow,f] = act(conv(x[n,h,w,c], w[kh,kw,c,f]) + bias[f]), implicit GEMM.
    `workspace` (optional, zero-filled, conv_workspace_bytes) enables the split-K tail.

    BatchNorm epilogues (inference form, reference conv2d_bn / conv2d_bn_relu /
    conv_bn_add_relu): bn = (gamma, beta, mean, var), [f] vectors of one dtype, replaces
    bias: out = act(bn(conv) [+ residual]); `residual` ([n,oh,ow,f], the output dtype)
    needs relu=True and clamps var at 0, as conv_bn_add_relu does."""
    dev = _require_cuda(x, w, bias, out, workspace, residual, *(bn or ()))
    if x.dim() != 4 or w.dim() != 4 or not x.is_contiguous() or not w.is_contiguous():
        raise ValueError("x must be contiguous NHWC [n,h,w,c] and w contiguous [kh,kw,c,f]")
    if x.dtype != w.dtype or x.dtype not in (torch.float16, torch.bfloat16):
        raise ValueError("x and w must share dtype float16 or bfloat16")
    n, h, wd, c = x.shape
    kh, kw, cw, f = w.shape
    if cw != c:
        raise ValueError(f"channel mismatch: x has C={c}, w has C={cw}")
    oh = (h + 2 * padding - dilation * (kh - 1) - 1) // stride + 1
    ow = (wd + 2 * padding - dilation * (kw - 1) - 1) // stride + 1
    if out is None:
        out = torch.empty((n, oh, ow, f), device=dev, dtype=out_dtype or x.dtype)
    if tuple(out.shape) != (n, oh, ow, f) or not out.is_contiguous():
        raise ValueError(f"out must be contiguous [{n},{oh},{ow},{f}]")
    bias = _vec(bias, f, "bias")
    if bn is not None:
        if bias is not None:
            raise ValueError("bn replaces bias: pass one of them")
        if len(bn) != 4:
            raise ValueError("bn must be (gamma, beta, mean, var)")
        bn = tuple(_vec(v, f, name) for v, name in zip(bn, ("gamma", "beta", "mean", "var")))
        if len({v.dtype for v in bn}) != 1:
            raise ValueError("gamma, beta, mean and var must share one dtype")
        if residual is not None:
            if not relu:
                raise ValueError("the residual epilogue is BN + add + ReLU: pass relu=True")
            if tuple(residual.shape) != (n, oh, ow, f) or residual.dtype != out.dtype or not residual.is_contiguous():
                raise ValueError(f"residual must be a contiguous [{n},{oh},{ow},{f}] tensor of {out.dtype}")
            epi = N.FO_EPI_BN_ADD_RELU
        else:
            epi = N.FO_EPI_BN_RELU if relu else N.FO_EPI_BN
    elif residual is not None:
        raise ValueError("a residual needs the BatchNorm epilogue (bn=...)")
    else:
        epi = {(False, False): N.FO_EPI_NONE, (True, False): N.FO_EPI_BIAS,
               (False, True): N.FO_EPI_RELU, (True, True): N.FO_EPI_BIAS_RELU}[(bias is not None, relu)]
    d = N.FoConvDesc()
    d.n, d.h, d.w, d.c, d.f, d.kh, d.kw = n, h, wd, c, f, kh, kw
    d.stride, d.pad, d.dil = stride, padding, dilation
    d.x, d.wgt, d.out = x.data_ptr(), w.data_ptr(), out.data_ptr()
    d.bias = bias.data_ptr() if bias is not None else None
    d.in_dtype, d.out_dtype = dtype_code(x.dtype), dtype_code(out.dtype)
    d.vec_dtype = dtype_code(bias.dtype) if bias is not None else N.FO_DT_F32
    if bn is not None:
        d.bn_gamma, d.bn_beta, d.bn_mean, d.bn_var = (v.data_ptr() for v in bn)
        d.bn_eps = bn_eps
        d.vec_dtype = dtype_code(bn[0].dtype)
        d.residual = residual.data_ptr() if residual is not None else None
    d.epilogue = epi
    cfg = as_tile_cfg(config) if config is not None else default_conv_config(f)
    if workspace is not None:
        d.workspace, d.workspace_bytes = workspace.data_ptr(), workspace.numel() * workspace.element_size()
    with torch.cuda.device(dev):
        N.check(N.lib().fo_conv2d(ctypes.byref(d), ctypes.byref(cfg), _stream(dev, stream)))
    return out
