"""Python host mirror of the llm-runner attention operator surface, on B200.

The reference records its attention ops through `RenderGraph.dispatch`
(lib/vulkan/graph.c3:47-72) with fp32 `llm::Tensor` bindings and a push
constant struct per op (dependencies/zimage.c3l/dit.c3:120-170). This package
exposes the same operators, with the same names, argument meaning and
argument order, over the C-ABI library `libllmr_attn.so` (include/llmr_attn.h):

    flash_attention_v2(ctx, q, k, v, o, head_dim, n_heads, seq_len, scale)
    batch_head_norm(ctx, data, gain, n_heads, head_dim, seq_len, eps)
    perhead_rmsnorm(ctx, data, weight, seq_len, n_heads, head_dim, eps)
    transpose_heads(ctx, inp, out, seq_len, n_heads, head_dim, direction)
    mrope(ctx, data, cos, sin, seq_len, n_heads)
    spatial_attention(ctx, q, k, v, scores, o, head_dim, n_heads, seq_len, scale)
    vae_attention(ctx, q, k, v, o, head_dim, n_heads, seq_len, scale, channels)
    split_qkv(ctx, qkv, q, k, v, dim, n_rows)

plus the fused op `attention_fused` that replaces the whole 8-dispatch
sequence of a DiT attention block. Buffers are torch CUDA tensors (device
memory and streams only; all compute is in the library's CUDA kernels).
There is no CPU fallback: importing this package without the built library
raises, and every op on a machine without an sm_100 GPU fails with
LlmrError(LLMR_ENODEV).
"""
from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass
from typing import Optional, Sequence

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
# LLMR_LIB may name another build of the same library (e.g. the diagnostic
# timeline build, `make TIMELINE=1 OUT=...`).
LIB_PATH = os.environ.get("LLMR_LIB") or os.path.join(os.path.dirname(_HERE), "libllmr_attn.so")

OK, EINVAL, ENOMEM, ECUDA, ENCCL, ETIMEOUT, ENODEV = range(7)
_STATUS_NAMES = {0: "LLMR_OK", 1: "LLMR_EINVAL", 2: "LLMR_ENOMEM", 3: "LLMR_ECUDA",
                 4: "LLMR_ENCCL", 5: "LLMR_ETIMEOUT", 6: "LLMR_ENODEV"}

F32, F16, BF16 = 0, 1, 2
BSHD, BHSD = 0, 1
NORM_Q, NORM_K, ROPE, EXACT, LSE, MERGE = 1, 2, 4, 8, 16, 32


class LlmrError(RuntimeError):
    """A non-zero status from the C ABI (the reference raises a fault)."""

    def __init__(self, status: int, message: str = ""):
        self.status = status
        super().__init__(f"{_STATUS_NAMES.get(status, status)}: {message}")


class AttnDesc(ctypes.Structure):
    """Mirror of llmr_attn_desc (include/llmr_attn.h)."""

    _fields_ = [
        ("batch", ctypes.c_uint32), ("n_heads", ctypes.c_uint32),
        ("seq_len", ctypes.c_uint32), ("head_dim", ctypes.c_uint32),
        ("in_dtype", ctypes.c_int), ("out_dtype", ctypes.c_int),
        ("layout", ctypes.c_int), ("flags", ctypes.c_uint32),
        ("scale", ctypes.c_float), ("eps", ctypes.c_float),
        ("split_row", ctypes.c_uint32), ("rope_row_offset", ctypes.c_uint32),
        ("q_row_stride", ctypes.c_uint64), ("k_row_stride", ctypes.c_uint64),
        ("v_row_stride", ctypes.c_uint64), ("o_row_stride", ctypes.c_uint64),
        ("q_batch_stride", ctypes.c_uint64), ("k_batch_stride", ctypes.c_uint64),
        ("v_batch_stride", ctypes.c_uint64), ("o_batch_stride", ctypes.c_uint64),
        ("q_head_stride", ctypes.c_uint64), ("k_head_stride", ctypes.c_uint64),
        ("v_head_stride", ctypes.c_uint64),
        ("kv_seq_len", ctypes.c_uint32),
    ]


class QkvDesc(ctypes.Structure):
    """llmr_qkv_desc (include/llmr_attn.h)."""
    _fields_ = [
        ("batch", ctypes.c_uint32), ("seq_len", ctypes.c_uint32),
        ("hidden", ctypes.c_uint32), ("n_heads", ctypes.c_uint32),
        ("head_dim", ctypes.c_uint32), ("dtype", ctypes.c_int), ("flags", ctypes.c_uint32),
        ("eps", ctypes.c_float), ("split_row", ctypes.c_uint32),
        ("rope_row_offset", ctypes.c_uint32), ("x_row_stride", ctypes.c_uint64),
    ]


class ProjDesc(ctypes.Structure):
    """llmr_proj_desc (include/llmr_attn.h)."""
    _fields_ = [
        ("batch", ctypes.c_uint32), ("seq_len", ctypes.c_uint32),
        ("in_dim", ctypes.c_uint32), ("out_dim", ctypes.c_uint32),
        ("dtype", ctypes.c_int), ("split_row", ctypes.c_uint32),
        ("o_row_stride", ctypes.c_uint64), ("hidden_row_stride", ctypes.c_uint64),
    ]


class IpcHandle(ctypes.Structure):
    """llmr_ipc_handle: an exported device allocation (64 opaque bytes)."""
    _fields_ = [("bytes", ctypes.c_ubyte * 64)]


def _load() -> ctypes.CDLL:
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"{LIB_PATH} is not built; run `make -C llm-runner_b200/csrc` "
            "(or __graft_entry__.build()). There is no CPU fallback.")
    lib = ctypes.CDLL(LIB_PATH)
    vp, u32, u64, f32, i32 = (ctypes.c_void_p, ctypes.c_uint32, ctypes.c_uint64,
                              ctypes.c_float, ctypes.c_int)
    sig = {
        "llmr_ctx_create": (i32, [i32, ctypes.c_size_t, vp, ctypes.POINTER(vp)]),
        "llmr_ctx_destroy": (i32, [vp]),
        "llmr_ctx_reserve": (i32, [vp, ctypes.c_size_t]),
        "llmr_set_stream": (i32, [vp, vp]),
        "llmr_ctx_set_sm_budget": (i32, [vp, i32]),
        "llmr_timeline_set": (i32, [vp, vp, ctypes.c_size_t]),
        "llmr_get_stream": (vp, [vp]),
        "llmr_last_error": (ctypes.c_char_p, [vp]),
        "llmr_sync": (i32, [vp]),
        "llmr_launch_count": (u64, [vp]),
        "llmr_selftest_wait_timeout": (i32, [vp, u64]),
        "llmr_profile_enable": (i32, [vp, i32]),
        "llmr_profile_read": (i32, [vp, ctypes.POINTER(ctypes.c_float)]),
        "llmr_alloc": (i32, [vp, ctypes.c_size_t, ctypes.POINTER(vp)]),
        "llmr_free": (i32, [vp, vp]),
        "llmr_upload": (i32, [vp, vp, vp, ctypes.c_size_t]),
        "llmr_download": (i32, [vp, vp, vp, ctypes.c_size_t]),
        "llmr_flash_attention_v2": (i32, [vp, vp, vp, vp, vp, u32, u32, u32, f32]),
        "llmr_batch_head_norm": (i32, [vp, vp, vp, u32, u32, u32, f32]),
        "llmr_perhead_rmsnorm": (i32, [vp, vp, vp, u32, u32, u32, f32]),
        "llmr_transpose_heads": (i32, [vp, vp, vp, u32, u32, u32, u32]),
        "llmr_mrope": (i32, [vp, vp, vp, vp, u32, u32]),
        "llmr_spatial_attention": (i32, [vp, vp, vp, vp, vp, vp, u32, u32, u32, f32]),
        "llmr_split_qkv": (i32, [vp, vp, vp, vp, vp, u32, u32]),
        "llmr_vae_attention": (i32, [vp, vp, vp, vp, vp, u32, u32, u32, f32, u32]),
        "llmr_attention_workspace_bytes": (ctypes.c_size_t, [ctypes.POINTER(AttnDesc)]),
        "llmr_attention_fused": (i32, [vp, ctypes.POINTER(AttnDesc), vp, vp, vp, vp, vp,
                                       vp, vp, vp, vp]),
        "llmr_attention_merge": (i32, [vp, vp, vp, vp, vp, u32, u32, u32, u64]),
        "llmr_attention_prologue": (i32, [vp, ctypes.POINTER(AttnDesc), vp, vp, vp, vp, vp,
                                          vp, vp, vp]),
        "llmr_convert_f32": (i32, [vp, vp, vp, ctypes.c_int, ctypes.c_size_t]),
        "llmr_attention_fused_noalloc": (i32, [ctypes.POINTER(AttnDesc), vp, vp, vp, vp, vp,
                                               vp, vp, vp, vp, vp]),
        "llmr_noalloc_status": (i32, [vp]),
        "llmr_rope_tables": (i32, [vp, u32, u32, vp, f32, vp, vp]),
        "llmr_qkv_project": (i32, [vp, ctypes.POINTER(QkvDesc), vp, vp, vp, vp, vp, vp, vp]),
        "llmr_attention_varlen": (i32, [vp, ctypes.POINTER(AttnDesc), vp, u32, vp, vp, vp, vp,
                                        vp, vp, vp, vp, vp]),
        "llmr_out_project": (i32, [vp, ctypes.POINTER(ProjDesc), vp, vp, vp, vp, vp, vp, vp,
                                   vp]),
        "llmr_ipc_export": (i32, [vp, vp, ctypes.POINTER(IpcHandle)]),
        "llmr_ipc_open": (i32, [vp, ctypes.POINTER(IpcHandle), ctypes.POINTER(vp)]),
        "llmr_ipc_close": (i32, [vp, vp]),
        "llmr_copy_async": (i32, [vp, vp, vp, ctypes.c_size_t, vp]),
        "llmr_copy2d_async": (i32, [vp, vp, ctypes.c_size_t, vp, ctypes.c_size_t,
                                    ctypes.c_size_t, ctypes.c_size_t, vp]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


lib = _load()


def _ptr(t) -> Optional[int]:
    """Device (or host numpy) address of a tensor/array; None passes NULL."""
    if t is None:
        return None
    if isinstance(t, np.ndarray):
        return t.ctypes.data
    return t.data_ptr()


class Context:
    """One llmr_ctx: a device, a CUDA stream, and a workspace.

    By default the context runs on torch's current stream of `device`, so
    library kernels and torch copies are ordered with each other and CUDA
    events recorded by torch time them. Replaces createContext()
    (lib/vulkan/context.c3:73).
    """

    def __init__(self, device: int = 0, workspace_bytes: int = 0, stream=None):
        import torch
        if stream is None:
            stream = torch.cuda.current_stream(device)
        handle = ctypes.c_void_p()
        raw = stream.cuda_stream if hasattr(stream, "cuda_stream") else stream
        if not raw:
            # torch's default stream is the legacy default stream (handle 0);
            # name it explicitly (cudaStreamLegacy) so that the library does
            # not create a stream of its own.
            raw = 1
        rc = lib.llmr_ctx_create(device, workspace_bytes, ctypes.c_void_p(raw),
                                 ctypes.byref(handle))
        if rc != OK:
            raise LlmrError(rc, f"llmr_ctx_create(device={device})")
        self.handle = handle
        self.device = device

    def check(self, rc: int) -> None:
        if rc != OK:
            msg = lib.llmr_last_error(self.handle)
            raise LlmrError(rc, msg.decode() if msg else "")

    def reserve(self, nbytes: int) -> None:
        self.check(lib.llmr_ctx_reserve(self.handle, nbytes))

    def timeline(self, buf) -> None:
        """Diagnostic builds: per-CTA event timestamps of the attention kernel
        into `buf` (a uint64/int64 CUDA tensor of >= num_sms * 64 elements;
        None turns it off)."""
        nbytes = 0 if buf is None else buf.numel() * buf.element_size()
        self.check(lib.llmr_timeline_set(self.handle, _ptr(buf), nbytes))

    def set_sm_budget(self, sms: int) -> None:
        """Persistent kernels of this context use at most `sms` SMs (0 = all)."""
        self.check(lib.llmr_ctx_set_sm_budget(self.handle, sms))

    def sync(self) -> None:
        self.check(lib.llmr_sync(self.handle))

    def profile(self, on: bool = True) -> None:
        """Per-phase CUDA-event timing of fused calls (prologue, attention)."""
        self.check(lib.llmr_profile_enable(self.handle, 1 if on else 0))

    def profile_read(self):
        """(prologue_ms, attention_ms) of the last profiled fused call."""
        ms = (ctypes.c_float * 2)()
        self.check(lib.llmr_profile_read(self.handle, ms))
        return float(ms[0]), float(ms[1])

    @property
    def launches(self) -> int:
        return int(lib.llmr_launch_count(self.handle))

    def close(self) -> None:
        if getattr(self, "handle", None):
            lib.llmr_ctx_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


# ---------------------------------------------------------------- reference op mirrors

def flash_attention_v2(ctx: Context, q, k, v, o, head_dim: int, n_heads: int,
                       seq_len: int, scale: float) -> None:
    """flash_attn.slang:38-241. q,k,v fp32 [H,S,D]; o fp32 [S,H*D]."""
    ctx.check(lib.llmr_flash_attention_v2(ctx.handle, _ptr(q), _ptr(k), _ptr(v), _ptr(o),
                                          head_dim, n_heads, seq_len, scale))


def batch_head_norm(ctx: Context, data, gain, n_heads: int, head_dim: int,
                    seq_len: int, eps: float) -> None:
    """zimage.slang:623-659, in place on fp32 [S,H*D]."""
    ctx.check(lib.llmr_batch_head_norm(ctx.handle, _ptr(data), _ptr(gain), n_heads,
                                       head_dim, seq_len, eps))


def perhead_rmsnorm(ctx: Context, data, weight, seq_len: int, n_heads: int,
                    head_dim: int, eps: float) -> None:
    """vit.slang:590-616, in place on fp32 [S,H*D]."""
    ctx.check(lib.llmr_perhead_rmsnorm(ctx.handle, _ptr(data), _ptr(weight), seq_len,
                                       n_heads, head_dim, eps))


def transpose_heads(ctx: Context, inp, out, seq_len: int, n_heads: int,
                    head_dim: int, direction: int) -> None:
    """zimage.slang:575-601: 0 = [S,H,D]->[H,S,D], 1 = reverse."""
    ctx.check(lib.llmr_transpose_heads(ctx.handle, _ptr(inp), _ptr(out), seq_len,
                                       n_heads, head_dim, direction))


def mrope(ctx: Context, data, cos, sin, seq_len: int, n_heads: int) -> None:
    """mrope.slang:33-54, in place on fp32 [H,S,128] with tables [S,64]."""
    ctx.check(lib.llmr_mrope(ctx.handle, _ptr(data), _ptr(cos), _ptr(sin), seq_len,
                             n_heads))


def spatial_attention(ctx: Context, q, k, v, scores, o, head_dim: int, n_heads: int,
                      seq_len: int, scale: float) -> None:
    """diffusion.slang:478-569; `scores` is accepted and ignored (may be None)."""
    ctx.check(lib.llmr_spatial_attention(ctx.handle, _ptr(q), _ptr(k), _ptr(v),
                                         _ptr(scores), _ptr(o), head_dim, n_heads,
                                         seq_len, scale))


def vae_attention(ctx: Context, q, k, v, o, head_dim: int, n_heads: int, seq_len: int,
                  scale: float, channels: int = 0) -> None:
    """diffusion.slang:1828-1975. q,k,v,o fp32 [S, C] (C = channels, default
    n_heads*head_dim), head h at columns [h*D, (h+1)*D); head_dim 64, 128,
    384 or 512. Tensor cores with fp16 operands; needs a workspace of
    3*S*H*D*2 bytes (ctx.reserve)."""
    channels = channels or n_heads * head_dim
    ctx.check(lib.llmr_vae_attention(ctx.handle, _ptr(q), _ptr(k), _ptr(v), _ptr(o),
                                     head_dim, n_heads, seq_len, scale, channels))


def split_qkv(ctx: Context, qkv, q, k, v, dim: int, n_rows: int) -> None:
    """depth.slang:40-58."""
    ctx.check(lib.llmr_split_qkv(ctx.handle, _ptr(qkv), _ptr(q), _ptr(k), _ptr(v), dim,
                                 n_rows))


# ------------------------------------------------------------------------ fused op

_TORCH_DTYPE_CODE = None


def _dtype_code(t) -> int:
    import torch
    table = {torch.float32: F32, torch.float16: F16, torch.bfloat16: BF16}
    if t.dtype not in table:
        raise LlmrError(EINVAL, f"unsupported dtype {t.dtype}")
    return table[t.dtype]


@dataclass
class AttnConfig:
    """Per-call parameters of the fused op (the push constants of the eight
    reference dispatches folded together)."""

    n_heads: int
    head_dim: int
    scale: float
    layout: int = BSHD
    eps: float = 1e-6
    norm_q: bool = False
    norm_k: bool = False
    rope: bool = False
    exact: bool = False
    split_row: int = 0
    rope_row_offset: int = 0


def make_desc(cfg: AttnConfig, batch: int, seq_len: int, in_dtype: int, out_dtype: int,
              lse: bool = False, strides: Optional[dict] = None,
              merge: bool = False, kv_len: int = 0) -> AttnDesc:
    d = AttnDesc()
    d.batch, d.n_heads, d.seq_len, d.head_dim = batch, cfg.n_heads, seq_len, cfg.head_dim
    d.kv_seq_len = kv_len
    d.in_dtype, d.out_dtype, d.layout = in_dtype, out_dtype, cfg.layout
    d.flags = ((NORM_Q if cfg.norm_q else 0) | (NORM_K if cfg.norm_k else 0)
               | (ROPE if cfg.rope else 0) | (EXACT if cfg.exact else 0)
               | (LSE if lse else 0) | (MERGE if merge else 0))
    d.scale, d.eps = cfg.scale, cfg.eps
    d.split_row, d.rope_row_offset = cfg.split_row, cfg.rope_row_offset
    for key, val in (strides or {}).items():
        setattr(d, key, int(val))
    return d


def workspace_bytes(desc: AttnDesc) -> int:
    return int(lib.llmr_attention_workspace_bytes(ctypes.byref(desc)))


def attention_fused(ctx: Context, q, k, v, o, cfg: AttnConfig, *, batch: int, seq_len: int,
                    q_gain=None, k_gain=None, cos=None, sin=None, lse=None,
                    strides: Optional[dict] = None, merge: bool = False,
                    kv_len: int = 0) -> None:
    """Fused QK-RMSNorm + RoPE + non-causal attention into `o` [B,S,H*D].

    q/k/v: torch CUDA tensors (f32/f16/bf16) in cfg.layout; gains fp32
    [D] or [2,D] (txt/img split at cfg.split_row); cos/sin fp32 [rows, D/2].
    merge: o (fp32) and lse already hold a result over other keys; this
    call's result is merged into them by log-sum-exp.
    kv_len: keys per (b, h) when not seq_len (fp16 q/k/v without norm/RoPE).
    """
    desc = make_desc(cfg, batch, seq_len, _dtype_code(q), _dtype_code(o),
                     lse=lse is not None, strides=strides, merge=merge, kv_len=kv_len)
    ctx.check(lib.llmr_attention_fused(ctx.handle, ctypes.byref(desc), _ptr(q), _ptr(k),
                                       _ptr(v), _ptr(q_gain), _ptr(k_gain), _ptr(cos),
                                       _ptr(sin), _ptr(o), _ptr(lse)))


def attention_varlen(ctx: Context, q, k, v, o, cfg: AttnConfig, seq_lens, *, q_gain=None,
                     k_gain=None, cos=None, sin=None, lse=None,
                     strides: Optional[dict] = None) -> None:
    """Packed variable-length sequences (llmr_attention_varlen): q/k/v/o hold
    len(seq_lens) sequences back to back as one batch element of
    sum(seq_lens) tokens; each attends within itself. cos/sin rows follow the
    packed token index (concatenated tables); no txt/img split."""
    lens = (ctypes.c_uint32 * len(seq_lens))(*[int(x) for x in seq_lens])
    tokens = q.shape[-3] if cfg.layout == BSHD else q.shape[-2]
    if tokens != int(sum(seq_lens)):
        raise LlmrError(EINVAL, f"seq_lens sum to {int(sum(seq_lens))}, q holds {tokens} tokens")
    desc = make_desc(cfg, 1, int(sum(seq_lens)), _dtype_code(q), _dtype_code(o),
                     lse=lse is not None, strides=strides)
    ctx.check(lib.llmr_attention_varlen(ctx.handle, ctypes.byref(desc), lens, len(seq_lens),
                                        _ptr(q), _ptr(k), _ptr(v), _ptr(q_gain), _ptr(k_gain),
                                        _ptr(cos), _ptr(sin), _ptr(o), _ptr(lse)))


NOALLOC_SCRATCH_BYTES = 64 << 20


def attention_fused_noalloc(q, k, v, o, cfg: AttnConfig, *, batch: int, seq_len: int,
                            q_gain=None, k_gain=None, cos=None, sin=None, lse=None,
                            strides: Optional[dict] = None, stream=None) -> None:
    """The allocation-free fused op (llmr_attention_fused_noalloc): no
    context, no device allocation; scratch is a fixed array inside the
    library (NOALLOC_SCRATCH_BYTES per GPU). For callers whose device memory
    is owned by another allocator or who must not call cudaMalloc/cudaFree.
    Runs on the current device, on `stream` (default: torch's current)."""
    import torch
    if stream is None:
        stream = torch.cuda.current_stream()
    raw = stream.cuda_stream if hasattr(stream, "cuda_stream") else stream
    desc = make_desc(cfg, batch, seq_len, _dtype_code(q), _dtype_code(o),
                     lse=lse is not None, strides=strides)
    rc = lib.llmr_attention_fused_noalloc(ctypes.byref(desc), _ptr(q), _ptr(k), _ptr(v),
                                          _ptr(q_gain), _ptr(k_gain), _ptr(cos), _ptr(sin),
                                          _ptr(o), _ptr(lse), ctypes.c_void_p(raw or None))
    if rc != OK:
        raise LlmrError(rc, "llmr_attention_fused_noalloc")


def noalloc_status(stream=None) -> None:
    """Synchronises `stream` and raises LlmrError(ETIMEOUT) if a bounded
    device-side wait of an allocation-free call on the current device expired
    since the last query (llmr_noalloc_status; the flag is cleared)."""
    import torch
    if stream is None:
        stream = torch.cuda.current_stream()
    raw = stream.cuda_stream if hasattr(stream, "cuda_stream") else stream
    rc = lib.llmr_noalloc_status(ctypes.c_void_p(raw or None))
    if rc != OK:
        raise LlmrError(rc, "llmr_noalloc_status")


def attention_prologue(ctx: Context, q, k, v, qkv_out, cfg: AttnConfig, *, batch: int,
                       seq_len: int, q_gain=None, k_gain=None, cos=None, sin=None,
                       strides: Optional[dict] = None) -> None:
    """Norm + RoPE of Q/K and cast of V into dense fp16 [3][B][H][S][D]."""
    desc = make_desc(cfg, batch, seq_len, _dtype_code(q), F16, strides=strides)
    ctx.check(lib.llmr_attention_prologue(ctx.handle, ctypes.byref(desc), _ptr(q), _ptr(k),
                                          _ptr(v), _ptr(q_gain), _ptr(k_gain), _ptr(cos),
                                          _ptr(sin), _ptr(qkv_out)))


def convert_f32(ctx: Context, src, dst) -> None:
    """dst <- src (fp32) converted to dst's dtype with RNE."""
    ctx.check(lib.llmr_convert_f32(ctx.handle, _ptr(src), _ptr(dst), _dtype_code(dst),
                                   src.numel()))


def attention_merge(ctx: Context, o_a, lse_a, o_b, lse_b, rows: int, n_heads: int,
                    head_dim: int, o_row_stride: int = 0) -> None:
    """(o_a, lse_a) <- LSE-merge of two partial results over disjoint keys."""
    ctx.check(lib.llmr_attention_merge(ctx.handle, _ptr(o_a), _ptr(lse_a), _ptr(o_b),
                                       _ptr(lse_b), rows, n_heads, head_dim, o_row_stride))


# -------------------------------------------------------------- QKV projection

def qkv_project(ctx: Context, x, w, qkv_out, cfg: AttnConfig, *, batch: int, seq_len: int,
                q_gain=None, k_gain=None, cos=None, sin=None) -> None:
    """qkv_out (fp16 [3, B, H, S, D]) <- x [B*S, hidden] . w[3*H*D, hidden]^T
    with cfg's RMSNorm (norm_q / norm_k, eps, split_row) and RoPE
    (rope, rope_row_offset) applied to Q and K in the epilogue. x and w are
    both fp16 or both bf16. The result feeds attention_fused with
    layout=BHSD, fp16 inputs and no norm/RoPE flags."""
    d = QkvDesc()
    d.batch, d.seq_len, d.hidden = batch, seq_len, x.shape[-1]
    d.n_heads, d.head_dim = cfg.n_heads, cfg.head_dim
    d.dtype = _dtype_code(x)
    d.flags = ((NORM_Q if cfg.norm_q else 0) | (NORM_K if cfg.norm_k else 0)
               | (ROPE if cfg.rope else 0))
    d.eps, d.split_row, d.rope_row_offset = cfg.eps, cfg.split_row, cfg.rope_row_offset
    d.x_row_stride = x.stride(-2) if x.dim() >= 2 else 0
    if _dtype_code(w) != d.dtype:
        raise LlmrError(EINVAL, "x and w must have the same dtype")
    ctx.check(lib.llmr_qkv_project(ctx.handle, ctypes.byref(d), _ptr(x), _ptr(w),
                                   _ptr(q_gain), _ptr(k_gain), _ptr(cos), _ptr(sin),
                                   _ptr(qkv_out)))


def out_project(ctx: Context, o, hidden, w0, w1=None, *, batch: int, seq_len: int,
                split_row: int = 0, bias0=None, bias1=None, gate0=None, gate1=None) -> None:
    """hidden (fp32 [B*S, out_dim]) += gate_g * (o . w_g^T + bias_g), weight
    set g = 1 for tokens >= split_row (when split_row > 0). o [B*S, in_dim]
    and the weights [out_dim, in_dim] are both fp16 or both bf16."""
    d = ProjDesc()
    d.batch, d.seq_len = batch, seq_len
    d.in_dim, d.out_dim = o.shape[-1], w0.shape[0]
    d.dtype = _dtype_code(o)
    d.split_row = split_row
    d.o_row_stride = o.stride(-2)
    d.hidden_row_stride = hidden.stride(-2)
    for w in (w0, w1):
        if w is not None and _dtype_code(w) != d.dtype:
            raise LlmrError(EINVAL, "o and the weights must have the same dtype")
    ctx.check(lib.llmr_out_project(ctx.handle, ctypes.byref(d), _ptr(o), _ptr(w0), _ptr(w1),
                                   _ptr(bias0), _ptr(bias1), _ptr(gate0), _ptr(gate1),
                                   _ptr(hidden)))


# --------------------------------------------------------------------- peer buffers

_TYPESTR = {"float16": "<f2", "bfloat16": None, "float32": "<f4", "uint8": "|u1"}


class DeviceBuffer:
    """A device allocation of its own (llmr_alloc), as IPC export needs, with
    torch views of it. Freed by close()."""

    def __init__(self, ctx: Context, nbytes: int):
        p = ctypes.c_void_p()
        ctx.check(lib.llmr_alloc(ctx.handle, nbytes, ctypes.byref(p)))
        self.ctx, self.ptr, self.nbytes = ctx, p.value, nbytes

    def tensor(self, shape, dtype):
        """A torch tensor over the whole buffer (dense, `shape`, `dtype`)."""
        import torch
        name = str(dtype).replace("torch.", "")
        n = int(np.prod(shape)) * torch.empty((), dtype=dtype).element_size()
        if _TYPESTR.get(name) is None or n > self.nbytes:
            raise LlmrError(EINVAL, f"cannot view {self.nbytes} bytes as {shape} {dtype}")
        view = _CudaArray(self.ptr, tuple(int(x) for x in shape), _TYPESTR[name])
        return torch.as_tensor(view, device=f"cuda:{self.ctx.device}")

    def export(self) -> bytes:
        h = IpcHandle()
        self.ctx.check(lib.llmr_ipc_export(self.ctx.handle, ctypes.c_void_p(self.ptr),
                                           ctypes.byref(h)))
        return bytes(h.bytes)

    def close(self) -> None:
        if self.ptr:
            self.ctx.check(lib.llmr_free(self.ctx.handle, ctypes.c_void_p(self.ptr)))
            self.ptr = None


class _CudaArray:
    def __init__(self, ptr, shape, typestr):
        self.__cuda_array_interface__ = {"data": (ptr, False), "shape": shape,
                                         "typestr": typestr, "version": 2}


class PeerMapping:
    """Another process's DeviceBuffer mapped into this one (llmr_ipc_open):
    `ptr` is readable by copies on this GPU."""

    def __init__(self, ctx: Context, handle: bytes):
        h = IpcHandle()
        ctypes.memmove(h.bytes, handle, 64)
        p = ctypes.c_void_p()
        ctx.check(lib.llmr_ipc_open(ctx.handle, ctypes.byref(h), ctypes.byref(p)))
        self.ctx, self.ptr = ctx, p.value

    def close(self) -> None:
        if self.ptr:
            self.ctx.check(lib.llmr_ipc_close(self.ctx.handle, ctypes.c_void_p(self.ptr)))
            self.ptr = None


def copy_async(ctx: Context, dst: int, src: int, nbytes: int, stream=None) -> None:
    """nbytes from address src to address dst on `stream` (copy engines; any
    two GPUs of the process, peer mappings included)."""
    raw = None
    if stream is not None:
        raw = stream.cuda_stream if hasattr(stream, "cuda_stream") else stream
    ctx.check(lib.llmr_copy_async(ctx.handle, ctypes.c_void_p(dst), ctypes.c_void_p(src),
                                  nbytes, ctypes.c_void_p(raw or None)))


def copy2d_async(ctx: Context, dst: int, dpitch: int, src: int, spitch: int, width: int,
                 height: int, stream=None) -> None:
    """`height` rows of `width` bytes between strided row sets (copy engines)."""
    raw = None
    if stream is not None:
        raw = stream.cuda_stream if hasattr(stream, "cuda_stream") else stream
    ctx.check(lib.llmr_copy2d_async(ctx.handle, ctypes.c_void_p(dst), dpitch,
                                    ctypes.c_void_p(src), spitch, width, height,
                                    ctypes.c_void_p(raw or None)))


# ------------------------------------------------------------------- host helpers

def rope_tables(pos: np.ndarray, axes_dims: Sequence[int], theta: float):
    """Multi-axis RoPE tables (flux_dit.c3:396-525, dit.c3:561-757), on the host.

    pos: int32 [S, n_axes]. Returns (cos, sin) float32 [S, sum(axes)/2].
    """
    pos = np.ascontiguousarray(pos, dtype=np.int32)
    axes = np.ascontiguousarray(axes_dims, dtype=np.uint32)
    S, n_axes = pos.shape
    if n_axes != len(axes):
        raise LlmrError(EINVAL, "pos columns != number of axes")
    half = int(axes.sum()) // 2
    cos = np.empty((S, half), np.float32)
    sin = np.empty((S, half), np.float32)
    rc = lib.llmr_rope_tables(pos.ctypes.data, S, n_axes, axes.ctypes.data, theta,
                              cos.ctypes.data, sin.ctypes.data)
    if rc != OK:
        raise LlmrError(rc, "llmr_rope_tables")
    return cos, sin


__all__ = [
    "Context", "LlmrError", "AttnConfig", "AttnDesc", "make_desc", "workspace_bytes",
    "flash_attention_v2", "batch_head_norm", "perhead_rmsnorm", "transpose_heads",
    "mrope", "spatial_attention", "vae_attention", "split_qkv", "attention_fused",
    "attention_merge", "rope_tables", "DeviceBuffer", "PeerMapping", "copy_async",
    "copy2d_async", "qkv_project", "QkvDesc", "out_project", "ProjDesc", "attention_varlen",
    "IpcHandle", "LIB_PATH", "lib",
]
