"""Python operators over the C ABI: the drop-in for the reference's hot path.

* ``attention(q, k, v, causal=False)`` on ``[B, H, S, D]`` CUDA tensors (bf16,
  fp16, or contiguous fp32 staged to bf16 on the device) --
  the operator behind the reference's kernel-module protocol (``bench.py:14-20``;
  ``pytorch-naive.py:23-65``, ``flash-attn2-sota.py:41-63``,
  ``old/kernels/old/naive.py:27-56``).
* ``attention_f32(q, k, v, k_transposed=False)`` -- the reference's own 2-D
  fp32 problem (``fn(KT, Q, V)``), staged to bf16 on the device in one call.
* ``attention_bshd(q, k, v, causal=False)`` -- the legacy ``(B, S, H, D)``
  layout of ``old/benchmark.py:17-21``, passed to the kernel as strides (no
  permute copy).
* ``mlp(x, w1, w2)`` -- ``act(x @ w1) @ w2``, the GEMM -> activation -> GEMM of
  ``run_mlp_search.py:58-69`` with the activation fused into GEMM 1.
* ``gemm_act(a, b, act)`` -- one matmul stage with its fused epilogue.
* ``mlp_ln(x, w1, w2)`` -- the reference's whole MLP block,
  ``LayerNorm(relu(x @ w1) @ w2 + x)`` (``run_mlp_search.py:42-127``).
* ``attention_from_host(...)`` / ``mlp_from_host(...)`` -- the same
  operators fed from (pinned) host tensors: copies in, kernels, copies out,
  pipelined over streams.

Errors: argument problems Python can see (device, dtype, rank) raise
``TypeError``/``ValueError``; everything the C ABI rejects raises
``FaError`` (a ``RuntimeError``) carrying ``fa_strerror``'s text, the way the
reference's modules surface failures as exceptions that ``bench.py:68-74``
records.  There is no CPU fallback.
"""

from __future__ import annotations

import ctypes
import math

import torch

from . import _lib

_BF16 = torch.bfloat16
_F16 = torch.float16
_HALF_TYPES = (_BF16, _F16)


# torch's raw current-stream accessor (the one its compiled kernels use) is
# ~10x cheaper than torch.cuda.current_stream(); small calls are host bound.
_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def _stream_ptr(device: torch.device) -> int:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    if _raw_stream is not None:
        return _raw_stream(idx)
    return torch.cuda.current_stream(idx).cuda_stream


# bf16 staging workspaces of attention_f32 up to this size are kept per
# (device, stream) and reused; work on one stream is ordered, so a reused
# workspace is never written while an earlier call still reads it.
_WS_CACHE_MAX_ELEMS = 8 << 20
_ws_cache: dict = {}


def _staging_workspace(n_elems: int, device: torch.device, stream: int) -> torch.Tensor:
    if n_elems > _WS_CACHE_MAX_ELEMS:
        return torch.empty(n_elems, dtype=_BF16, device=device)
    key = (device.index, stream)
    ws = _ws_cache.get(key)
    if ws is None or ws.numel() < n_elems:
        if ws is None and len(_ws_cache) >= 16:
            # Many streams: drop the cache (torch's allocator reuses a freed
            # block only for work on the stream it was allocated on).
            _ws_cache.clear()
        ws = torch.empty(max(n_elems, 1 << 16), dtype=_BF16, device=device)
        _ws_cache[key] = ws
    return ws


class _on_device:
    """Make ``device`` current for the C call (the library launches on the
    current device); a no-op when it already is, which keeps small calls cheap."""

    __slots__ = ("idx", "prev")

    def __init__(self, device: torch.device):
        self.idx = device.index if device.index is not None else torch.cuda.current_device()
        self.prev = None

    def __enter__(self):
        cur = torch.cuda.current_device()
        if cur != self.idx:
            self.prev = cur
            torch.cuda.set_device(self.idx)
        return self

    def __exit__(self, *exc):
        if self.prev is not None:
            torch.cuda.set_device(self.prev)


def _check_cuda(name: str, t: torch.Tensor, dtypes=(_BF16,)) -> None:
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor")
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor (got device {t.device})")
    if t.dtype not in dtypes:
        names = " or ".join(str(d).replace("torch.", "") for d in dtypes)
        raise TypeError(f"{name} must be {names} (got {t.dtype})")


def _check_cuda_bf16(name: str, t: torch.Tensor) -> None:
    _check_cuda(name, t, (_BF16,))


def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool = False,
              scale: float | None = None, out: torch.Tensor | None = None,
              precise: bool = False) -> torch.Tensor:
    """softmax(q k^T * scale [+ causal mask]) v on ``[B, H, S, D]`` CUDA tensors.

    ``scale`` defaults to ``1/sqrt(D)`` (``run_attention_search.py:40``); D is
    8 .. 128, a multiple of 8.  bf16 and fp16 inputs (all three the same
    type) run the tensor cores in that type with fp32 accumulation; they may
    have arbitrary batch/head/sequence strides (multiples of 8 elements) but
    must be contiguous along D.  fp32 inputs (the reference's dtype) must be
    contiguous; they are staged to bf16 on the device in the same C call and
    O is written in fp32.  With ``precise`` (fp32 inputs, D <= 64) every
    operand is staged as a bf16 hi + lo pair and the GEMMs take the three
    significant products (about 16 significant bits instead of 8, three times
    the tensor-core work).  Returns a new ``[B, H, S, D]`` tensor of the input
    dtype unless ``out`` is given.
    """
    for name, t in (("q", q), ("k", k), ("v", v)):
        _check_cuda(name, t, (_BF16, _F16, torch.float32))
        if t.dim() != 4:
            raise ValueError(f"{name} must be 4-D [B, H, S, D] (got {tuple(t.shape)})")
    if not (q.shape == k.shape == v.shape):
        raise ValueError(f"q, k, v shapes differ: {tuple(q.shape)}, {tuple(k.shape)}, "
                         f"{tuple(v.shape)}")
    if not (q.dtype == k.dtype == v.dtype):
        raise TypeError(f"q, k, v dtypes differ: {q.dtype}, {k.dtype}, {v.dtype}")
    if not (q.device == k.device == v.device):
        raise ValueError("q, k, v must be on the same device")
    B, H, S, D = q.shape
    dtype = q.dtype
    if out is None:
        out = torch.empty((B, H, S, D), dtype=dtype, device=q.device)
    else:
        _check_cuda("out", out, (dtype,))
        if tuple(out.shape) != (B, H, S, D) or out.device != q.device:
            raise ValueError("out must match q's shape and device")
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    if B * H * S == 0:
        return out                 # empty batch, heads or sequence: nothing to compute
    lib = _lib.load()
    if dtype == torch.float32:
        for name, t in (("q", q), ("k", k), ("v", v), ("out", out)):
            if not t.is_contiguous():
                raise ValueError(f"fp32 {name} must be contiguous")
        mode = _lib.FA_F32_SPLIT if precise else _lib.FA_F32_BF16
        width = 128 if precise else D
        with _on_device(q.device):
            stream = _stream_ptr(q.device)
            ws = _staging_workspace(3 * B * H * S * width, q.device, stream)
            rc = lib.fa_attn_fwd_f32_batched(q.data_ptr(), k.data_ptr(), v.data_ptr(),
                                             out.data_ptr(), ws.data_ptr(), B, H, S, D, 0,
                                             int(bool(causal)), float(scale), mode, stream)
        _lib.check(rc, "fa_attn_fwd_f32_batched")
        return out
    if precise:
        raise ValueError("precise applies to fp32 inputs")
    strides = (ctypes.c_int64 * 16)(*q.stride(), *k.stride(), *v.stride(), *out.stride())
    fn, where = ((lib.fa_attn_fwd_f16, "fa_attn_fwd_f16") if dtype == _F16
                 else (lib.fa_attn_fwd, "fa_attn_fwd"))
    with _on_device(q.device):
        rc = fn(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), B, H, S, D, strides,
                int(bool(causal)), float(scale), _stream_ptr(q.device))
    _lib.check(rc, where)
    return out


def attention_f32(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool = False,
                  scale: float | None = None, k_transposed: bool = False,
                  out: torch.Tensor | None = None, precise: bool = False) -> torch.Tensor:
    """The reference's own 2-D fp32 problem: ``q [N, D]``, ``k [N, D]`` (or
    ``KT [D, N]`` with ``k_transposed=True``), ``v [N, D]`` contiguous fp32
    CUDA tensors -> ``o [N, D]`` fp32.  One C call: the operands are staged to
    bf16 on the device and the attention epilogue writes fp32 (the
    ``fn(KT, Q, V)`` of ``pytorch-naive.py:23`` and the emitted modules).
    ``precise`` stages bf16 hi + lo pairs instead (D <= 64), see ``attention``."""
    for name, t in (("q", q), ("k", k), ("v", v)):
        if not isinstance(t, torch.Tensor):
            raise TypeError(f"{name} must be a torch.Tensor")
        if not t.is_cuda:
            raise ValueError(f"{name} must be a CUDA tensor (got device {t.device})")
        if t.dtype != torch.float32:
            raise TypeError(f"{name} must be float32 (got {t.dtype})")
        if t.dim() != 2 or not t.is_contiguous():
            raise ValueError(f"{name} must be a contiguous 2-D tensor")
    N, D = q.shape
    kshape = (D, N) if k_transposed else (N, D)
    if tuple(v.shape) != (N, D) or tuple(k.shape) != kshape:
        raise ValueError(f"shapes q {tuple(q.shape)}, k {tuple(k.shape)}, v {tuple(v.shape)} "
                         f"do not match (k expected {kshape})")
    if not (q.device == k.device == v.device):
        raise ValueError("q, k, v must be on the same device")
    if out is None:
        out = torch.empty((N, D), dtype=torch.float32, device=q.device)
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    lib = _lib.load()
    with _on_device(q.device):
        stream = _stream_ptr(q.device)
        if precise:
            ws = _staging_workspace(3 * N * 128, q.device, stream)
            rc = lib.fa_attn_fwd_f32_batched(q.data_ptr(), k.data_ptr(), v.data_ptr(),
                                             out.data_ptr(), ws.data_ptr(), 1, 1, N, D,
                                             int(bool(k_transposed)), int(bool(causal)),
                                             float(scale), _lib.FA_F32_SPLIT, stream)
            where = "fa_attn_fwd_f32_batched"
        else:
            ws = _staging_workspace(3 * N * D, q.device, stream)
            rc = lib.fa_attn_fwd_f32(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(),
                                     ws.data_ptr(), N, D, int(bool(k_transposed)),
                                     int(bool(causal)), float(scale), stream)
            where = "fa_attn_fwd_f32"
    _lib.check(rc, where)
    return out


def attention_bshd(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool = False,
                   scale: float | None = None) -> torch.Tensor:
    """The legacy ``fn(q, k, v)`` on ``(B, S, H, D)`` bf16 or fp16 tensors
    (``old/benchmark.py:17-21``, fp16 by default there); the head/sequence
    transpose is expressed as strides, so no data is copied.  Returns
    ``(B, S, H, D)``."""
    for name, t in (("q", q), ("k", k), ("v", v)):
        _check_cuda(name, t, _HALF_TYPES)
        if t.dim() != 4:
            raise ValueError(f"{name} must be 4-D (B, S, H, D)")
    out = torch.empty_like(q, memory_format=torch.contiguous_format)
    attention(q.permute(0, 2, 1, 3), k.permute(0, 2, 1, 3), v.permute(0, 2, 1, 3),
              causal=causal, scale=scale, out=out.permute(0, 2, 1, 3))
    return out


def attention_from_host(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                        causal: bool = False, scale: float | None = None,
                        out: torch.Tensor | None = None,
                        device: torch.device | int | str | None = None,
                        workspace: dict | None = None, chunks: int = 8) -> torch.Tensor:
    """``attention`` for ``[B, H, S, D]`` host tensors: host-to-device copy of
    q, k, v, the fused kernel, device-to-host copy of O.

    The (batch, head) pairs are split into ``chunks`` groups that flow through
    three streams -- copies in, kernel, copies out -- chained by events, so
    the two PCIe directions and the kernels overlap; the current stream of
    ``device`` waits for the last copy out, so work ordered after the call on
    that stream (or a synchronize) sees the whole result.  Host tensors should
    be pinned and contiguous for the copies to be asynchronous.  The result
    lands in ``out`` (allocated pinned if omitted).  ``workspace`` (a dict)
    keeps the device buffers, streams and events between calls.
    """
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None \
        else torch.device(device)
    if dev.type != "cuda":
        raise ValueError("device must be a CUDA device")
    for name, t in (("q", q), ("k", k), ("v", v)):
        if t.is_cuda or t.dtype not in _HALF_TYPES or t.dtype != q.dtype:
            raise ValueError(f"{name} must be a bfloat16 or float16 host tensor (all alike)")
        if t.dim() != 4 or not t.is_contiguous():
            raise ValueError(f"{name} must be a contiguous 4-D [B, H, S, D] tensor")
    B, H, S, D = q.shape
    dtype = q.dtype
    pairs = B * H
    nch = max(1, min(int(chunks), pairs))
    bounds = [pairs * i // nch for i in range(nch + 1)]
    ws = workspace if workspace is not None else {}
    key = (tuple(q.shape), dtype, dev, nch)
    if ws.get("key") != key:
        for st in ws.get("streams", ()):
            st.synchronize()          # the old buffers may still be in use
        ws.clear()
        ws["key"] = key
        for name in ("q", "k", "v", "o"):
            ws[name] = torch.empty((1, pairs, S, D), dtype=dtype, device=dev)
        ws["streams"] = [torch.cuda.Stream(device=dev) for _ in range(3)]
        ws["ev_in"] = [torch.cuda.Event() for _ in range(nch)]
        ws["ev_cmp"] = [torch.cuda.Event() for _ in range(nch)]
        ws["ev_out"] = torch.cuda.Event()
    if out is None:
        out = torch.empty(q.shape, dtype=dtype, pin_memory=True)
    s_in, s_cmp, s_out = ws["streams"]
    cur = torch.cuda.current_stream(dev)
    # the previous call's consumers of the buffers are ordered before us
    s_in.wait_stream(cur)
    s_cmp.wait_stream(cur)
    s_out.wait_stream(cur)
    hq, hk, hv, ho = (t.view(1, pairs, S, D) for t in (q, k, v, out))
    for c in range(nch):
        a, z = bounds[c], bounds[c + 1]
        with torch.cuda.stream(s_in):
            ws["q"][:, a:z].copy_(hq[:, a:z], non_blocking=True)
            ws["k"][:, a:z].copy_(hk[:, a:z], non_blocking=True)
            ws["v"][:, a:z].copy_(hv[:, a:z], non_blocking=True)
            ws["ev_in"][c].record(s_in)
        s_cmp.wait_event(ws["ev_in"][c])
        with torch.cuda.stream(s_cmp):
            attention(ws["q"][:, a:z], ws["k"][:, a:z], ws["v"][:, a:z], causal=causal,
                      scale=scale, out=ws["o"][:, a:z])
            ws["ev_cmp"][c].record(s_cmp)
        s_out.wait_event(ws["ev_cmp"][c])
        with torch.cuda.stream(s_out):
            ho[:, a:z].copy_(ws["o"][:, a:z], non_blocking=True)
    ws["ev_out"].record(s_out)
    cur.wait_event(ws["ev_out"])
    return out


def mlp_from_host(x: torch.Tensor, w1: torch.Tensor, w2: torch.Tensor,
                  act: str = "gelu_tanh", out: torch.Tensor | None = None,
                  workspace: dict | None = None, chunks: int = 4) -> torch.Tensor:
    """``mlp`` for a host ``x [M, K]`` with device-resident weights (the serving
    shape: weights loaded once, activations streamed): host-to-device copy of
    x, the two GEMMs, device-to-host copy of y.  The rows are split into
    ``chunks`` blocks (multiples of 128 rows) that flow through copy-in /
    compute / copy-out streams chained by events, so both PCIe directions
    overlap the GEMMs; the current stream waits for the last copy out.  Host
    tensors should be pinned; ``out`` is allocated pinned if omitted;
    ``workspace`` (a dict) keeps device buffers, streams and events."""
    _check_cuda_bf16("w1", w1)
    _check_cuda_bf16("w2", w2)
    if x.is_cuda or x.dtype != _BF16 or x.dim() != 2 or not x.is_contiguous():
        raise ValueError("x must be a contiguous 2-D bfloat16 host tensor")
    dev = w1.device
    M, K = x.shape
    N = w1.shape[1]
    tiles = (M + 127) // 128
    nch = max(1, min(int(chunks), tiles))
    bounds = [min(M, 128 * (tiles * i // nch)) for i in range(nch + 1)]
    ws = workspace if workspace is not None else {}
    key = (M, K, N, dev, nch)
    if ws.get("key") != key:
        for st in ws.get("streams", ()):
            st.synchronize()
        ws.clear()
        ws["key"] = key
        ws["x"] = torch.empty((M, K), dtype=_BF16, device=dev)
        ws["h"] = torch.empty((M, N), dtype=_BF16, device=dev)
        ws["y"] = torch.empty((M, K), dtype=_BF16, device=dev)
        ws["streams"] = [torch.cuda.Stream(device=dev) for _ in range(3)]
        ws["ev_in"] = [torch.cuda.Event() for _ in range(nch)]
        ws["ev_cmp"] = [torch.cuda.Event() for _ in range(nch)]
        ws["ev_out"] = torch.cuda.Event()
    if out is None:
        out = torch.empty((M, K), dtype=_BF16, pin_memory=True)
    s_in, s_cmp, s_out = ws["streams"]
    cur = torch.cuda.current_stream(dev)
    for st in (s_in, s_cmp, s_out):
        st.wait_stream(cur)
    for c in range(nch):
        a, z = bounds[c], bounds[c + 1]
        if a == z:
            continue
        with torch.cuda.stream(s_in):
            ws["x"][a:z].copy_(x[a:z], non_blocking=True)
            ws["ev_in"][c].record(s_in)
        s_cmp.wait_event(ws["ev_in"][c])
        with torch.cuda.stream(s_cmp):
            mlp(ws["x"][a:z], w1, w2, act=act, hidden=ws["h"][a:z], out=ws["y"][a:z])
            ws["ev_cmp"][c].record(s_cmp)
        s_out.wait_event(ws["ev_cmp"][c])
        with torch.cuda.stream(s_out):
            out[a:z].copy_(ws["y"][a:z], non_blocking=True)
    ws["ev_out"].record(s_out)
    cur.wait_event(ws["ev_out"])
    return out


def gemm_act(a: torch.Tensor, b: torch.Tensor, act: str = "none",
             out: torch.Tensor | None = None) -> torch.Tensor:
    """``act(a @ b)`` for row-major ``a [M, K]``, ``b [K, N]`` (both bf16 or
    both fp16; the result has their dtype); K and N multiples of 64."""
    _check_cuda("a", a, _HALF_TYPES)
    _check_cuda("b", b, (a.dtype,))
    if a.dim() != 2 or b.dim() != 2 or a.shape[1] != b.shape[0]:
        raise ValueError(f"bad GEMM shapes {tuple(a.shape)} @ {tuple(b.shape)}")
    if a.stride(1) != 1 or b.stride(1) != 1:
        raise ValueError("a and b must be row-major (last dimension contiguous)")
    if act not in _lib.ACTIVATIONS:
        raise ValueError(f"act must be one of {sorted(_lib.ACTIVATIONS)}")
    M, K = a.shape
    N = b.shape[1]
    if out is None:
        out = torch.empty((M, N), dtype=a.dtype, device=a.device)
    else:
        _check_cuda("out", out, (a.dtype,))
    if M == 0:
        return out                 # no rows: nothing to compute
    lib = _lib.load()
    fn, where = ((lib.fa_gemm_act_f16, "fa_gemm_act_f16") if a.dtype == _F16
                 else (lib.fa_gemm_act, "fa_gemm_act"))
    with _on_device(a.device):
        rc = fn(a.data_ptr(), b.data_ptr(), out.data_ptr(), M, N, K, a.stride(0), b.stride(0),
                out.stride(0), _lib.ACTIVATIONS[act], _stream_ptr(a.device))
    _lib.check(rc, where)
    return out


def mlp(x: torch.Tensor, w1: torch.Tensor, w2: torch.Tensor, act: str = "gelu_tanh",
        hidden: torch.Tensor | None = None, out: torch.Tensor | None = None) -> torch.Tensor:
    """``act(x @ w1) @ w2`` with ``x [M, K]``, ``w1 [K, N]``, ``w2 [N, K]``
    (row-major, all bf16 or all fp16, K and N multiples of 64).  ``act`` is
    "gelu_tanh" (the benchmark block) or "relu" (``run_mlp_search.py:62-64``).
    ``hidden`` is the ``[M, N]`` workspace for ``act(x @ w1)``."""
    _check_cuda("x", x, _HALF_TYPES)
    for name, t in (("x", x), ("w1", w1), ("w2", w2)):
        _check_cuda(name, t, (x.dtype,))
        if t.dim() != 2 or not t.is_contiguous():
            raise ValueError(f"{name} must be a contiguous 2-D tensor")
    M, K = x.shape
    if w1.shape[0] != K or w2.shape[1] != K or w2.shape[0] != w1.shape[1]:
        raise ValueError(f"bad MLP shapes x{tuple(x.shape)} w1{tuple(w1.shape)} "
                         f"w2{tuple(w2.shape)}")
    N = w1.shape[1]
    if act not in ("gelu_tanh", "relu"):
        raise ValueError("act must be 'gelu_tanh' or 'relu'")
    if hidden is None:
        hidden = torch.empty((M, N), dtype=x.dtype, device=x.device)
    if out is None:
        out = torch.empty((M, K), dtype=x.dtype, device=x.device)
    _check_cuda("hidden", hidden, (x.dtype,))
    _check_cuda("out", out, (x.dtype,))
    if M == 0:
        return out                 # no rows: nothing to compute
    lib = _lib.load()
    fn, where = ((lib.fa_mlp_fwd_f16, "fa_mlp_fwd_f16") if x.dtype == _F16
                 else (lib.fa_mlp_fwd, "fa_mlp_fwd"))
    with _on_device(x.device):
        rc = fn(x.data_ptr(), w1.data_ptr(), w2.data_ptr(), hidden.data_ptr(), out.data_ptr(),
                M, K, N, _lib.ACTIVATIONS[act], _stream_ptr(x.device))
    _lib.check(rc, where)
    return out


def mlp_ln(x: torch.Tensor, w1: torch.Tensor, w2: torch.Tensor, eps: float = 1e-5,
           hidden: torch.Tensor | None = None, resid: torch.Tensor | None = None,
           out: torch.Tensor | None = None) -> torch.Tensor:
    """The reference's MLP block ``LayerNorm(relu(x @ w1) @ w2 + x)`` without
    affine parameters (``run_mlp_search.py:42-127``, oracle ``:138-149``):
    ReLU fused into GEMM 1, the residual add into GEMM 2's epilogue, then a
    row LayerNorm kernel.  ``hidden`` [M, N] and ``resid`` [M, K] are bf16
    workspaces; K <= 8192."""
    for name, t in (("x", x), ("w1", w1), ("w2", w2)):
        _check_cuda_bf16(name, t)
        if t.dim() != 2 or not t.is_contiguous():
            raise ValueError(f"{name} must be a contiguous 2-D tensor")
    M, K = x.shape
    if w1.shape[0] != K or w2.shape[1] != K or w2.shape[0] != w1.shape[1]:
        raise ValueError(f"bad MLP shapes x{tuple(x.shape)} w1{tuple(w1.shape)} "
                         f"w2{tuple(w2.shape)}")
    N = w1.shape[1]
    hidden = torch.empty((M, N), dtype=_BF16, device=x.device) if hidden is None else hidden
    resid = torch.empty((M, K), dtype=_BF16, device=x.device) if resid is None else resid
    out = torch.empty((M, K), dtype=_BF16, device=x.device) if out is None else out
    if M == 0:
        return out                 # no rows: nothing to compute
    lib = _lib.load()
    with _on_device(x.device):
        rc = lib.fa_mlp_ln_fwd(x.data_ptr(), w1.data_ptr(), w2.data_ptr(), hidden.data_ptr(),
                               resid.data_ptr(), out.data_ptr(), M, K, N, float(eps),
                               _stream_ptr(x.device))
    _lib.check(rc, "fa_mlp_ln_fwd")
    return out


def layer_norm_rows(x: torch.Tensor, eps: float = 1e-5,
                    out: torch.Tensor | None = None) -> torch.Tensor:
    """``(x - mean) / sqrt(var + eps)`` over the last dimension of a 2-D bf16
    CUDA tensor (no affine; N a multiple of 8, N <= 8192)."""
    _check_cuda_bf16("x", x)
    if x.dim() != 2 or x.stride(1) != 1:
        raise ValueError("x must be 2-D with a contiguous last dimension")
    M, N = x.shape
    out = torch.empty((M, N), dtype=_BF16, device=x.device) if out is None else out
    if M == 0:
        return out                 # no rows: nothing to compute
    lib = _lib.load()
    with _on_device(x.device):
        rc = lib.fa_layernorm_rows(x.data_ptr(), out.data_ptr(), M, N, x.stride(0),
                                   out.stride(0), float(eps), _stream_ptr(x.device))
    _lib.check(rc, "fa_layernorm_rows")
    return out


def device_status() -> int:
    """Read and clear the device-side status word (FA_OK or FA_ERR_TIMEOUT)."""
    return _lib.load().fa_device_status()
