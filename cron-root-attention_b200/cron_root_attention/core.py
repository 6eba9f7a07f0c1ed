"""Functional API and autograd Function of the B200 sqrt(N) sparse attention.

Mirrors ``cron_root_attention/core.py`` of the reference package:
  * ``cron_root_attention_v14(q, k, v, use_persistent=False, kv_groups=1,
    relay_log_scale=None, relay_top_k=2)`` (reference core.py:3767-3797),
  * ``CronRootAttentionV14Function`` (reference core.py:2822-3759),
  * ``cron_root_attention_varlen`` / ``warmup_varlen_shapes``
    (reference core.py:3836-4022),
  * ``get_num_sms`` / ``GPU_SM_MAP`` (reference core.py:58-188).

All computation runs in libcra (hand-written sm_100a kernels, include/cra.h).
There is no Triton, no backend dispatch and no CPU fallback: CPU tensors
raise.  Semantics kept from the reference: W = ceil(sqrt(S)) (core.py:3479);
the relay phase is skipped for S <= 2048 (core.py:2832,3507); top-k exact
relay tokens by ||k||^2 (core.py:2630-2748); optional per-head relay scale
exp(relay_log_scale) (core.py:3541-3544).

Input handling: fp16 / bf16 run natively; fp32 inputs are computed in bf16
and the results returned in fp32.  head_dim 64 and 128 run natively; smaller
head dims are zero-padded to 64 (96..127 to 128) with the softmax scale of the
true head_dim, which leaves scores and outputs unchanged.
"""
from __future__ import annotations

import ctypes
import math
import os
from functools import lru_cache
from typing import Optional, Sequence, Union

import torch

from . import _lib
from ._lib import check, lib, strides3

RELAY_THRESHOLD = 2048

# SM counts by device name (reference core.py:58-140).  Used only when the
# device does not report its own count.  B200 has 148 SMs.
GPU_SM_MAP = {
    "NVIDIA B200": 148,
    "NVIDIA B100": 132,
    "NVIDIA GB200": 152,
    "NVIDIA H100 SXM": 132,
    "NVIDIA H100 PCIe": 114,
    "NVIDIA H200": 132,
    "NVIDIA A100 SXM": 108,
    "NVIDIA GeForce RTX 5090": 170,
    "NVIDIA GeForce RTX 5070 Ti": 70,
}


@lru_cache(maxsize=None)
def _sm_count(device_index: int) -> int:
    return torch.cuda.get_device_properties(device_index).multi_processor_count


def get_num_sms() -> int:
    """SM count of the current CUDA device (1 without CUDA); reference core.py:142-171."""
    if not torch.cuda.is_available():
        return 1
    n = _sm_count(torch.cuda.current_device())
    if n > 0:
        return n
    name = torch.cuda.get_device_name()
    for known, cnt in GPU_SM_MAP.items():
        if known in name or name in known:
            return cnt
    return 48


# ---------------------------------------------------------------------------
# per-device error word: kernels record a timed-out wait here instead of
# trapping; ``check_device_errors`` reads it.  A kernel that gave up on a wait
# leaves its outputs partly written, so a caller that cannot rule that out
# polls ``check_device_errors`` at a convenient point (for example once per
# training step), or sets CRA_CHECK_DEVICE_ERRORS=1 to have every forward and
# backward call synchronize and raise RuntimeError when the word is set.
_ERR_WORDS: dict = {}
_CHECK_EACH_CALL = os.environ.get("CRA_CHECK_DEVICE_ERRORS", "0") not in ("", "0")


def _err_word(device: torch.device) -> torch.Tensor:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    t = _ERR_WORDS.get(idx)
    if t is None:
        t = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", idx))
        _ERR_WORDS[idx] = t
    return t


def check_device_errors(device: Optional[torch.device] = None, reset: bool = True) -> int:
    """Return (and by default clear) the device error word of ``device``.
    0 = no kernel gave up on a bounded wait since the last check; 1
    (CRA_DEV_WAIT_TIMEOUT) = some kernel did, and the outputs of the calls
    since the last check are not to be trusted.  Reading the word
    synchronizes the device."""
    device = device or torch.device("cuda", torch.cuda.current_device())
    t = _err_word(device)
    v = int(t.item())
    if reset and v:
        t.zero_()
    return v


def _raise_on_device_error(device: torch.device, what: str) -> None:
    """With CRA_CHECK_DEVICE_ERRORS set: synchronize and raise when a kernel of
    ``what`` (or an earlier unchecked call) gave up on a bounded wait."""
    if _CHECK_EACH_CALL:
        code = check_device_errors(device)
        if code:
            raise RuntimeError(f"cron_root_attention {what}: a kernel gave up on a bounded device wait "
                               f"(device error {code}); its outputs are incomplete")


def _dtype_code(dt: torch.dtype) -> int:
    return _lib.CRA_BF16 if dt == torch.bfloat16 else _lib.CRA_F16


def _prep(x: torch.Tensor, cdt: torch.dtype, Dp: int) -> torch.Tensor:
    """Cast to the compute dtype, zero-pad head_dim to Dp, make TMA-legal."""
    if x.dtype != cdt:
        x = x.to(cdt)
    D = x.shape[-1]
    if D != Dp:
        x = torch.nn.functional.pad(x, (0, Dp - D))
    if x.stride(-1) != 1 or any(s % 8 for s in x.stride()[:3]) or x.data_ptr() % 16:
        x = x.contiguous()
    return x


def _padded_dim(D: int) -> int:
    if D <= 64:
        return 64
    if D <= 128:
        return 128
    raise NotImplementedError(f"head_dim {D} > 128 is not supported")


def _stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _launch_fwd(L, qc, kc, vc, gk, gv, gsrc, alpha, B, Hq, Hkv, S, Dp, cdt, use_relay, relay_top_k, scale,
                dev, stream):
    """relay build + forward kernel through the C ABI; returns (o, lse)."""
    check(L.cra_relay_build(kc.data_ptr(), vc.data_ptr(), strides3(kc), strides3(vc),
                            B, Hkv, S, Dp, _dtype_code(cdt), use_relay, relay_top_k,
                            alpha.data_ptr() if alpha is not None else None,
                            gk.data_ptr(), gv.data_ptr(), gsrc.data_ptr(), stream), "cra_relay_build")
    o = torch.empty(B, Hq, S, Dp, device=dev, dtype=cdt)
    lse = torch.empty(B, Hq, S, device=dev, dtype=torch.float32)
    check(L.cra_fwd(qc.data_ptr(), kc.data_ptr(), vc.data_ptr(), gk.data_ptr(), gv.data_ptr(),
                    strides3(qc), strides3(kc), strides3(vc), B, Hq, Hkv, S, Dp, _dtype_code(cdt),
                    use_relay, relay_top_k, ctypes.c_float(scale), o.data_ptr(), strides3(o),
                    lse.data_ptr(), _err_word(dev).data_ptr(), stream), "cra_fwd")
    return o, lse


class CronRootAttentionV14Function(torch.autograd.Function):
    """Autograd Function; same forward arguments as the reference
    (core.py:3472-3476) and the same gradient tuple shape (core.py:3759)."""

    RELAY_THRESHOLD = RELAY_THRESHOLD

    @staticmethod
    def forward(ctx, q, k, v, use_persistent=False, kv_groups=1, relay_log_scale=None, relay_top_k=2):
        if not (q.is_cuda and k.is_cuda and v.is_cuda):
            raise RuntimeError("cron_root_attention: tensors must be on a CUDA device (no CPU fallback)")
        if q.dim() != 4 or k.dim() != 4 or v.dim() != 4:
            raise ValueError("q, k, v must be [B, H, S, D]")
        B, Hq, S, D = q.shape
        Hkv = k.shape[1]
        if k.shape != v.shape or k.shape[0] != B or k.shape[2] != S or k.shape[3] != D:
            raise ValueError(f"shape mismatch q{tuple(q.shape)} k{tuple(k.shape)} v{tuple(v.shape)}")
        if Hkv * kv_groups != Hq:
            raise ValueError(f"kv_groups={kv_groups} inconsistent with H_q={Hq}, H_kv={Hkv}")
        if not 1 <= relay_top_k <= 4:
            raise ValueError("relay_top_k must be in 1..4")
        dev = q.device
        in_dtype = q.dtype
        cdt = in_dtype if in_dtype in (torch.float16, torch.bfloat16) else torch.bfloat16
        Dp = _padded_dim(D)
        scale = 1.0 / math.sqrt(D)
        L = lib()
        use_relay = int(S > RELAY_THRESHOLD)
        qc, kc, vc = (_prep(t, cdt, Dp) for t in (q, k, v))
        NG = L.cra_global_rows(S, use_relay, relay_top_k)
        NB = (S + L.cra_window(S) - 1) // L.cra_window(S)
        gk = torch.empty(B, Hkv, NG, Dp, device=dev, dtype=cdt)
        gv = torch.empty_like(gk)
        gsrc = torch.empty(B, Hkv, NB, relay_top_k, device=dev, dtype=torch.int32)
        alpha = None
        if relay_log_scale is not None and use_relay:
            alpha = relay_log_scale.detach().to(device=dev, dtype=torch.float32).contiguous()
            if alpha.numel() != Hkv:
                raise ValueError("relay_log_scale must have H_kv elements")
        stream = _stream_ptr(dev)
        with torch.cuda.device(dev):
            o, lse = _launch_fwd(L, qc, kc, vc, gk, gv, gsrc, alpha, B, Hq, Hkv, S, Dp, cdt, use_relay,
                                 relay_top_k, scale, dev, stream)
        _raise_on_device_error(dev, "forward")
        ctx.save_for_backward(qc, kc, vc, o, lse, gk, gv, gsrc, alpha)
        ctx.meta = (B, Hq, Hkv, S, D, Dp, use_relay, relay_top_k, scale, in_dtype, cdt,
                    relay_log_scale is not None)
        out = o if Dp == D else o[..., :D]
        if out.dtype != in_dtype:
            out = out.to(in_dtype)
        return out

    @staticmethod
    def backward(ctx, do):
        qc, kc, vc, o, lse, gk, gv, gsrc, alpha = ctx.saved_tensors
        B, Hq, Hkv, S, D, Dp, use_relay, top_k, scale, in_dtype, cdt, has_alpha = ctx.meta
        dev = qc.device
        L = lib()
        doc = _prep(do, cdt, Dp)
        dq = torch.empty_like(qc)
        dk = torch.empty_like(kc)
        dv = torch.empty_like(vc)
        dalpha = torch.zeros(Hkv, device=dev, dtype=torch.float32) if alpha is not None else None
        ws_bytes = L.cra_bwd_workspace_bytes(B, Hq, Hkv, S, Dp, use_relay, top_k)
        ws = torch.empty(max(ws_bytes, 1), device=dev, dtype=torch.uint8)
        stream = _stream_ptr(dev)
        with torch.cuda.device(dev):
            check(L.cra_bwd(qc.data_ptr(), kc.data_ptr(), vc.data_ptr(), o.data_ptr(), doc.data_ptr(),
                            lse.data_ptr(), gk.data_ptr(), gv.data_ptr(), gsrc.data_ptr(),
                            strides3(qc), strides3(kc), strides3(vc), strides3(o), strides3(doc),
                            B, Hq, Hkv, S, Dp, _dtype_code(cdt), use_relay, top_k, ctypes.c_float(scale),
                            alpha.data_ptr() if alpha is not None else None,
                            dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), strides3(dq), strides3(dk), strides3(dv),
                            dalpha.data_ptr() if dalpha is not None else None,
                            ws.data_ptr(), ws_bytes, _err_word(dev).data_ptr(), stream), "cra_bwd")
        _raise_on_device_error(dev, "backward")

        def fin(t):
            t = t if Dp == D else t[..., :D]
            return t if t.dtype == in_dtype else t.to(in_dtype)

        d_alpha = None
        if has_alpha:
            d_alpha = dalpha if dalpha is not None else torch.zeros(Hkv, device=dev, dtype=torch.float32)
        return fin(dq), fin(dk), fin(dv), None, None, d_alpha, None


@torch.compiler.disable
def cron_root_attention_v14(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                            use_persistent: bool = False, kv_groups: int = 1,
                            relay_log_scale: Optional[torch.Tensor] = None,
                            relay_top_k: int = 2) -> torch.Tensor:
    """Causal 3-phase sqrt(N) attention (reference core.py:3767-3797).

    q: [B, H_q, S, D]; k, v: [B, H_kv, S, D] with H_q = H_kv * kv_groups.
    ``use_persistent`` is accepted for API compatibility; the B200 kernels
    choose their own scheduling.  Returns [B, H_q, S, D] in q's dtype.
    """
    return CronRootAttentionV14Function.apply(q, k, v, use_persistent, kv_groups, relay_log_scale, relay_top_k)


cron_root_attention = cron_root_attention_v14


class _VarlenFunction(torch.autograd.Function):
    """Packed variable-length attention.  Forward: one relay-build launch and
    one attention launch for all documents (libcra's varlen entry points,
    driven by a device document table).  Backward: the documents are grouped
    by length and each group runs as one batched cra_bwd call (the global
    rows rebuilt from K, which gives the same rows the forward used)."""

    @staticmethod
    def forward(ctx, q, k, v, seqs, kv_groups, relay_log_scale, relay_top_k):
        if not (q.is_cuda and k.is_cuda and v.is_cuda):
            raise RuntimeError("cron_root_attention: tensors must be on a CUDA device (no CPU fallback)")
        B, Hq, T, D = q.shape
        Hkv = k.shape[1]
        if Hkv * kv_groups != Hq:
            raise ValueError(f"kv_groups={kv_groups} inconsistent with H_q={Hq}, H_kv={Hkv}")
        if not 1 <= relay_top_k <= 4:
            raise ValueError("relay_top_k must be in 1..4")
        dev = q.device
        in_dtype = q.dtype
        cdt = in_dtype if in_dtype in (torch.float16, torch.bfloat16) else torch.bfloat16
        Dp = _padded_dim(D)
        scale = 1.0 / math.sqrt(D)
        L = lib()
        qc, kc, vc = (_prep(t, cdt, Dp) for t in (q, k, v))
        nd = len(seqs) - 1
        cu = (ctypes.c_int64 * len(seqs))(*seqs)
        NG = L.cra_varlen_global_rows(cu, nd, relay_top_k)
        NBt = L.cra_varlen_blocks(cu, nd)
        table = torch.empty(max(L.cra_varlen_table_bytes(nd), 1), device=dev, dtype=torch.uint8)
        gk = torch.empty(B, Hkv, max(NG, 1), Dp, device=dev, dtype=cdt)
        gv = torch.empty_like(gk)
        gsrc = torch.empty(B, Hkv, max(NBt, 1), relay_top_k, device=dev, dtype=torch.int32)
        alpha = None
        if relay_log_scale is not None:
            alpha = relay_log_scale.detach().to(device=dev, dtype=torch.float32).contiguous()
            if alpha.numel() != Hkv:
                raise ValueError("relay_log_scale must have H_kv elements")
        o = torch.empty(B, Hq, T, Dp, device=dev, dtype=cdt)
        lse = torch.empty(B, Hq, T, device=dev, dtype=torch.float32)
        stream = _stream_ptr(dev)
        with torch.cuda.device(dev):
            check(L.cra_varlen_plan(cu, nd, relay_top_k, table.data_ptr(), stream), "cra_varlen_plan")
            check(L.cra_relay_build_varlen(kc.data_ptr(), vc.data_ptr(), strides3(kc), strides3(vc), B, Hkv, cu, nd,
                                           table.data_ptr(), Dp, _dtype_code(cdt), relay_top_k,
                                           alpha.data_ptr() if alpha is not None else None, gk.data_ptr(),
                                           gv.data_ptr(), gsrc.data_ptr(), stream), "cra_relay_build_varlen")
            check(L.cra_fwd_varlen(qc.data_ptr(), kc.data_ptr(), vc.data_ptr(), gk.data_ptr(), gv.data_ptr(),
                                   strides3(qc), strides3(kc), strides3(vc), B, Hq, Hkv, cu, nd, table.data_ptr(), Dp,
                                   _dtype_code(cdt), relay_top_k, ctypes.c_float(scale), o.data_ptr(), strides3(o),
                                   lse.data_ptr(), _err_word(dev).data_ptr(), stream), "cra_fwd_varlen")
        _raise_on_device_error(dev, "varlen forward")
        ctx.save_for_backward(qc, kc, vc, o, lse, alpha)
        ctx.meta = (seqs, kv_groups, relay_top_k, D, Dp, scale, in_dtype, cdt, relay_log_scale is not None)
        out = o if Dp == D else o[..., :D]
        return out if out.dtype == in_dtype else out.to(in_dtype)

    @staticmethod
    def backward(ctx, do):
        qc, kc, vc, o, lse, alpha = ctx.saved_tensors
        seqs, kv_groups, top_k, D, Dp, scale, in_dtype, cdt, has_alpha = ctx.meta
        dev = qc.device
        L = lib()
        B, Hq, T, _ = qc.shape
        Hkv = kc.shape[1]
        doc_ = _prep(do, cdt, Dp)
        dq = torch.zeros_like(qc)
        dk = torch.zeros_like(kc)
        dv = torch.zeros_like(vc)
        dalpha = torch.zeros(Hkv, device=dev, dtype=torch.float32) if alpha is not None else None
        groups = {}
        for s0, s1 in zip(seqs, seqs[1:]):
            groups.setdefault(s1 - s0, []).append(s0)
        stream = _stream_ptr(dev)
        for n, starts in groups.items():
            def stack(t):
                if len(starts) == 1:
                    return _prep(t.narrow(2, starts[0], n), cdt, Dp)
                return torch.cat([t.narrow(2, s0, n) for s0 in starts], dim=0)
            qg, kg, vg, og, dog = (stack(t) for t in (qc, kc, vc, o, doc_))
            lg = torch.cat([lse.narrow(2, s0, n) for s0 in starts], dim=0).contiguous()
            G = B * len(starts)
            use_relay = int(n > RELAY_THRESHOLD)
            NG = L.cra_global_rows(n, use_relay, top_k)
            NB = (n + L.cra_window(n) - 1) // L.cra_window(n)
            gk = torch.empty(G, Hkv, NG, Dp, device=dev, dtype=cdt)
            gv = torch.empty_like(gk)
            gsrc = torch.empty(G, Hkv, NB, top_k, device=dev, dtype=torch.int32)
            a_g = alpha if (alpha is not None and use_relay) else None
            dqg, dkg, dvg = torch.empty_like(qg), torch.empty_like(kg), torch.empty_like(vg)
            da = torch.zeros(Hkv, device=dev, dtype=torch.float32) if a_g is not None else None
            ws_bytes = L.cra_bwd_workspace_bytes(G, Hq, Hkv, n, Dp, use_relay, top_k)
            ws = torch.empty(max(ws_bytes, 1), device=dev, dtype=torch.uint8)
            with torch.cuda.device(dev):
                check(L.cra_relay_build(kg.data_ptr(), vg.data_ptr(), strides3(kg), strides3(vg), G, Hkv, n, Dp,
                                        _dtype_code(cdt), use_relay, top_k,
                                        a_g.data_ptr() if a_g is not None else None, gk.data_ptr(), gv.data_ptr(),
                                        gsrc.data_ptr(), stream), "cra_relay_build")
                check(L.cra_bwd(qg.data_ptr(), kg.data_ptr(), vg.data_ptr(), og.data_ptr(), dog.data_ptr(),
                                lg.data_ptr(), gk.data_ptr(), gv.data_ptr(), gsrc.data_ptr(), strides3(qg),
                                strides3(kg), strides3(vg), strides3(og), strides3(dog), G, Hq, Hkv, n, Dp,
                                _dtype_code(cdt), use_relay, top_k, ctypes.c_float(scale),
                                a_g.data_ptr() if a_g is not None else None, dqg.data_ptr(), dkg.data_ptr(),
                                dvg.data_ptr(), strides3(dqg), strides3(dkg), strides3(dvg),
                                da.data_ptr() if da is not None else None, ws.data_ptr(), ws_bytes,
                                _err_word(dev).data_ptr(), stream), "cra_bwd")
            for i, s0 in enumerate(starts):
                dq.narrow(2, s0, n).copy_(dqg.narrow(0, i * B, B))
                dk.narrow(2, s0, n).copy_(dkg.narrow(0, i * B, B))
                dv.narrow(2, s0, n).copy_(dvg.narrow(0, i * B, B))
            if da is not None:
                dalpha += da
        _raise_on_device_error(dev, "varlen backward")

        def fin(t):
            t = t if Dp == D else t[..., :D]
            return t if t.dtype == in_dtype else t.to(in_dtype)

        d_alpha = None
        if has_alpha:
            d_alpha = dalpha if dalpha is not None else torch.zeros(Hkv, device=dev, dtype=torch.float32)
        return fin(dq), fin(dk), fin(dv), None, None, d_alpha, None


@torch.compiler.disable
def cron_root_attention_varlen(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                               cu_seqlens: Union[Sequence[int], torch.Tensor], kv_groups: int = 1,
                               use_persistent: bool = False,
                               relay_log_scale: Optional[torch.Tensor] = None,
                               relay_top_k: int = 2) -> torch.Tensor:
    """Packed variable-length attention (reference core.py:3836-3954): each
    document [cu_seqlens[i], cu_seqlens[i+1]) of the packed sequence
    dimension attends only to itself, with its own window and relay switch.
    ``cu_seqlens`` must be a CPU tensor or a Python sequence.  The forward
    runs as one launch over (document, query tile, head) -- the reference
    makes one call per document; the backward runs one batched call per
    distinct document length."""
    if isinstance(cu_seqlens, torch.Tensor):
        if cu_seqlens.device.type != "cpu":
            raise ValueError("cu_seqlens must be a CPU tensor to avoid a device sync on each "
                             "document boundary read.  Call cu_seqlens.cpu() first.")
        seqs = [int(x) for x in cu_seqlens.tolist()]
    else:
        seqs = [int(x) for x in cu_seqlens]
    if len(seqs) < 2 or seqs[0] != 0 or seqs[-1] != q.shape[2] or any(b < a for a, b in zip(seqs, seqs[1:])):
        raise ValueError("cu_seqlens must start at 0, end at S_total and be non-decreasing")
    if len(seqs) == 2:
        return cron_root_attention_v14(q, k, v, use_persistent=use_persistent, kv_groups=kv_groups,
                                       relay_log_scale=relay_log_scale, relay_top_k=relay_top_k)
    docs = [seqs[0]] + [b for a, b in zip(seqs, seqs[1:]) if b > a]  # empty documents dropped
    return _VarlenFunction.apply(q, k, v, docs, kv_groups, relay_log_scale, relay_top_k)


def warmup_varlen_shapes(doc_lengths, H: int, D: int, dtype=None, kv_groups: int = 1,
                         device=None, verbose: bool = False) -> None:
    """Run one forward per distinct document length (reference core.py:3957-4022).
    The B200 kernels are compiled ahead of time, so this only warms the
    allocator and the driver's tensor-map path."""
    dtype = dtype or torch.float16
    device = device or torch.device("cuda", torch.cuda.current_device())
    for S in sorted(set(int(x) for x in doc_lengths)):
        q = torch.zeros(1, H, S, D, device=device, dtype=dtype)
        kv = torch.zeros(1, H // kv_groups, S, D, device=device, dtype=dtype)
        cron_root_attention_v14(q, kv, kv, kv_groups=kv_groups)
        if verbose:
            print(f"  warmed S={S}")
    torch.cuda.synchronize(device)
