"""Operators of the reference's decode path on torch CUDA tensors.

Names and argument meaning follow the kernels of src/engine.cu in
g023/cuda_inf (gemv_int4, rmsnorm, rope, kv_commit_group, ...); each call goes
through the C ABI of libcuinf.so on the current torch CUDA stream.  Tensors
must be CUDA and contiguous; fp16 activations, u8 packed INT4 / FP8, fp32
GEMV outputs.  Errors raise CuinfError; nothing falls back to the CPU.
"""
import ctypes

import torch

from ._lib import check, lib

__all__ = [
    "gemv_int4", "gemv_fp16", "rmsnorm", "rmsnorm_head", "rope", "kv_write_tail",
    "kv_commit_group", "attn_decode", "attn_decode_noalloc", "conv_pre", "conv_apply", "conv_update_state", "swiglu",
    "acc_scaled", "add_inplace", "add_f32_inplace", "f32_to_f16", "embed_gather", "argmax",
    "moe_route", "moe_ffn", "quantize_int4", "expert_table",
]


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _p(t):
    if t is None:
        return None
    if not t.is_cuda:
        raise ValueError("expected a CUDA tensor")
    if not t.is_contiguous():
        raise ValueError("expected a contiguous tensor")
    return ctypes.c_void_p(t.data_ptr())


def _dt(t, dtype, name):
    if t.dtype != dtype:
        raise TypeError(f"{name} must be {dtype}, got {t.dtype}")


def gemv_int4(x, packed, scales, y=None):
    """y[m,n] = sum_k x[m,k] * (nib-8) * scale[n,k/128]  (gemv_int4, engine.cu:83-109).

    x fp16 [M,K] (or [K]); packed u8 [N,K/2]; scales fp16 [N,K/128]; y fp32 [M,N]."""
    _dt(x, torch.float16, "x"), _dt(packed, torch.uint8, "packed"), _dt(scales, torch.float16, "scales")
    N, K = packed.shape[0], packed.shape[1] * 2
    M = x.numel() // K
    if y is None:
        y = torch.empty((M, N) if x.dim() > 1 else (N,), dtype=torch.float32, device=x.device)
    check(lib().cuinf_gemv_int4(_p(x), _p(packed), _p(scales), _p(y), M, N, K, _stream()))
    return y


def gemm_int4_tc(x, packed, scales, y=None):
    """Tensor-core form of gemv_int4 for M activation rows (tcgen05)."""
    _dt(x, torch.float16, "x"), _dt(packed, torch.uint8, "packed"), _dt(scales, torch.float16, "scales")
    N, K = packed.shape[0], packed.shape[1] * 2
    M = x.numel() // K
    if y is None:
        y = torch.empty((M, N), dtype=torch.float32, device=x.device)
    check(lib().cuinf_gemm_int4_tc(_p(x), _p(packed), _p(scales), _p(y), M, N, K, _stream()))
    return y


def gemm_fp16_tc(x, W, want_logits=True):
    """Tensor-core x[M,K] . W[N,K]^T with the fused argmax; returns
    (logits fp32 [M,N] or None, argmax int [M])."""
    _dt(x, torch.float16, "x"), _dt(W, torch.float16, "W")
    N, K = W.shape
    M = x.numel() // K
    y = torch.empty((M, N), dtype=torch.float32, device=x.device) if want_logits else None
    keys = torch.zeros(M, dtype=torch.int64, device=x.device)
    check(lib().cuinf_gemm_fp16_tc(_p(x), _p(W), _p(y) if y is not None else None, M, N, K, _p(keys),
                                   _stream()))
    idx = [lib().cuinf_argmax_key_index(int(k) & 0xFFFFFFFFFFFFFFFF) for k in keys.cpu().tolist()]
    return y, idx


def gemv_fp16(x, W, y=None):
    """y[m,n] = sum_k x[m,k] * W[n,k]  (gemv_fp16, engine.cu:112-128)."""
    _dt(x, torch.float16, "x"), _dt(W, torch.float16, "W")
    N, K = W.shape
    M = x.numel() // K
    if y is None:
        y = torch.empty((M, N) if x.dim() > 1 else (N,), dtype=torch.float32, device=x.device)
    check(lib().cuinf_gemv_fp16(_p(x), _p(W), _p(y), M, N, K, _stream()))
    return y


def rmsnorm(inp, w, out=None, eps=1e-5):
    """half(x * rsqrt(mean(x^2) + eps) * w) per row  (rmsnorm, engine.cu:131-144)."""
    D = w.numel()
    M = inp.numel() // D
    if out is None:
        out = torch.empty_like(inp)
    check(lib().cuinf_rmsnorm(_p(inp), _p(w), _p(out), M, D, eps, _stream()))
    return out


def rmsnorm_head(inp, w, out=None, eps=1e-5):
    """Per-head RMSNorm over head_dim 64  (rmsnorm_head, engine.cu:148-158)."""
    return rmsnorm(inp, w, out, eps)


def rope(q, k, pos, theta=5e6):
    """In-place NEOX RoPE on q [S,nq,64] and k [S,nk,64]  (rope, engine.cu:161-182)."""
    S = pos.numel()
    nq = q.numel() // (S * 64)
    nk = k.numel() // (S * 64) if k is not None else 0
    check(lib().cuinf_rope(_p(q), _p(k), _p(pos), S, nq, nk, theta, _stream()))


def kv_write_tail(k, v, ktail, vtail, slot, cnt):
    """Copy cnt tokens into the fp16 tail at slot  (kv_write_tail, engine.cu:190-198)."""
    nkv = ktail.shape[1]
    check(lib().cuinf_kv_write_tail(_p(k), _p(v), _p(ktail), _p(vtail), slot, cnt, nkv, _stream()))


def kv_commit_group(ktail, vtail, kc8, vc8, ksc, vsc, dst_tok_base, grp):
    """Commit a full 64-token tail to FP8 E4M3  (kv_commit_group, engine.cu:202-228)."""
    nkv = ktail.shape[1]
    check(lib().cuinf_kv_commit_group(_p(ktail), _p(vtail), _p(kc8), _p(vc8), _p(ksc), _p(vsc),
                                      dst_tok_base, grp, nkv, _stream()))


def attn_decode(q, kc8, vc8, ksc, vsc, ktail, vtail, committed, qpos, scale=0.125, out=None,
                workspace=None):
    """Flash-decoding attention of one token over FP8 groups + fp16 tail
    (attn_decode_split + attn_decode_combine, engine.cu:396-480).  q [nh,64]."""
    nh = q.numel() // 64
    nkv = ktail.shape[1]
    if out is None:
        out = torch.empty_like(q)
    ws_bytes = workspace.numel() * workspace.element_size() if workspace is not None else 0
    check(lib().cuinf_attn_decode(_p(q), _p(kc8), _p(vc8), _p(ksc), _p(vsc), _p(ktail), _p(vtail),
                                  committed, qpos, scale, _p(out), nh, nkv, _p(workspace), ws_bytes,
                                  _stream()))
    return out


def attn_decode_noalloc(q, kc8, vc8, ksc, vsc, ktail, vtail, committed, qpos, scale=0.125,
                        out=None):
    """attn_decode with the library's static 512 KiB scratch: the C call allocates
    no device memory (out is allocated here only when not given).  Calls on
    one device must not overlap."""
    nh = q.numel() // 64
    nkv = ktail.shape[1]
    if out is None:
        out = torch.empty_like(q)
    check(lib().cuinf_attn_decode_noalloc(_p(q), _p(kc8), _p(vc8), _p(ksc), _p(vsc), _p(ktail),
                                          _p(vtail), committed, qpos, scale, _p(out), nh, nkv,
                                          _stream()))
    return out


def conv_pre(inproj, C, Bx, S, H):
    """C = half(C), Bx = half(B*x) from in_proj rows B|C|x  (conv_pre, engine.cu:483-494)."""
    check(lib().cuinf_conv_pre(_p(inproj), _p(C), _p(Bx), S, H, _stream()))


def conv_apply(Bx, C, w, state, y, S, H):
    """Causal depthwise conv k=3 gated by C  (conv_apply, engine.cu:498-512)."""
    check(lib().cuinf_conv_apply(_p(Bx), _p(C), _p(w), _p(state), _p(y), S, H, _stream()))


def conv_update_state(Bx, state, S, H):
    """Keep the last two Bx  (conv_update_state, engine.cu:514-525)."""
    check(lib().cuinf_conv_update_state(_p(Bx), _p(state), S, H, _stream()))


def swiglu(g, u, out):
    """out = half(silu(g) * u)  (swiglu, engine.cu:542-547)."""
    check(lib().cuinf_swiglu(_p(g), _p(u), _p(out), g.numel(), _stream()))


def acc_scaled(dst, src, w):
    """dst = half(dst + w * src)  (acc_scaled, engine.cu:556-559)."""
    check(lib().cuinf_acc_scaled(_p(dst), _p(src), float(w), dst.numel(), _stream()))


def add_inplace(a, b):
    """a = half(a + b)  (add_inplace, engine.cu:527-530)."""
    check(lib().cuinf_add_inplace(_p(a), _p(b), a.numel(), _stream()))


def add_f32_inplace(a, b):
    """a = half(a + b_f32)  (add_f32_inplace, engine.cu:532-535)."""
    check(lib().cuinf_add_f32_inplace(_p(a), _p(b), a.numel(), _stream()))


def f32_to_f16(src, dst):
    """dst = half(src)  (f32_to_f16, engine.cu:537-540)."""
    check(lib().cuinf_f32_to_f16(_p(src), _p(dst), src.numel(), _stream()))


def embed_gather(embed, ids, out):
    """out[s,:] = embed[ids[s],:]  (embed_gather, engine.cu:549-554)."""
    H = embed.shape[1]
    check(lib().cuinf_embed_gather(_p(embed), _p(ids), _p(out), ids.numel(), H, _stream()))


def argmax(logits, out=None):
    """Index of the max logit with argmax_kernel's tie rule (engine.cu:562-572)."""
    if out is None:
        out = torch.empty(1, dtype=torch.int32, device=logits.device)
    check(lib().cuinf_argmax(_p(logits), logits.numel(), _p(out), _stream()))
    return out


def moe_route(logits, bias, topk, idx=None, w=None):
    """Sigmoid + expert bias, top-k, norm_topk_prob on the device
    (the host loop of engine.cu:883-892).  logits fp32 [S,E], bias fp16 [E]."""
    E = bias.numel()
    S = logits.numel() // E
    if idx is None:
        idx = torch.empty((S, topk), dtype=torch.int32, device=logits.device)
    if w is None:
        w = torch.empty((S, topk), dtype=torch.float32, device=logits.device)
    check(lib().cuinf_moe_route(_p(logits), _p(bias), S, E, topk, _p(idx), _p(w), _stream()))
    return idx, w


def expert_table(experts):
    """Device table of per-expert pointers for moe_ffn: experts is a list of
    (w1_packed, w1_scales, w3_packed, w3_scales, w2_packed, w2_scales)."""
    ptrs = [t.data_ptr() for e in experts for t in e]
    dev = experts[0][0].device
    return torch.tensor(ptrs, dtype=torch.int64, device=dev)


def moe_ffn(xn, gate, expert_bias, table, h, topk, moe_inter, idx=None, w=None):
    """Fused MoE FFN of one token, h updated in place (engine.cu:877-905)."""
    H = h.numel()
    E = expert_bias.numel()
    check(lib().cuinf_moe_ffn(_p(xn), _p(gate), _p(expert_bias), _p(table), _p(h), H, moe_inter, E,
                              topk, _p(idx), _p(w), None, 0, _stream()))


def quantize_int4(w):
    """INT4 G=128 export quantizer of tools/export_weights.py:64-79 on the device.

    w fp32 [N,K] CUDA -> (packed u8 [N,K/2], scales fp16 [N,K/128])."""
    _dt(w, torch.float32, "w")
    N, K = w.shape
    packed = torch.empty((N, K // 2), dtype=torch.uint8, device=w.device)
    scales = torch.empty((N, K // 128), dtype=torch.float16, device=w.device)
    check(lib().cuinf_quantize_int4(_p(w), N, K, _p(packed), _p(scales), _stream()))
    return packed, scales
