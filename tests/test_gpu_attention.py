"""Causal attention kernels (fer_attn_causal_ex) on the GPU.

Two kernels sit behind the entry point: the tcgen05 one (S a multiple of
128) and the mma.sync one (any S, or forced with flags bit 0). Both compute
softmax(q k^T / 8) v per head over the fused QKV activation with P rounded to
bf16 before P.V; the reference here is the same arithmetic in float32 torch
with a two-pass softmax.

Tolerance: TOL = 1e-2 of max |reference| (bf16 output and bf16 P, online vs
two-pass rescaling); the two kernels agree within the same bound, and each is
bit-identical run to run.
"""
import ctypes as C

import pytest
import torch

from fercuda_b200 import capi

pytestmark = pytest.mark.gpu

TOL = 1e-2


def attn(qkv, B, S, heads, flags):
    k = capi.kernels()
    k.fer_attn_causal_ex.argtypes = [C.c_void_p, C.c_void_p] + [C.c_int] * 5 + [C.c_void_p, C.c_void_p]
    k.fer_attn_causal_ex.restype = C.c_int
    d = heads * 64
    out = torch.full((B * S, d), float("nan"), dtype=torch.bfloat16, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    rc = k.fer_attn_causal_ex(qkv.data_ptr(), out.data_ptr(), B, S, d, heads, flags, err.data_ptr(),
                              torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    return out


def reference(qkv, B, S, heads):
    d = heads * 64
    x = qkv.float().view(B, S, 3, heads, 64)
    q, k, v = (x[:, :, i].transpose(1, 2) for i in range(3))          # [B, h, S, 64]
    s = (q @ k.transpose(-1, -2)) / 8.0
    s = s.masked_fill(torch.triu(torch.ones(S, S, dtype=torch.bool, device=qkv.device), 1), float("-inf"))
    p = torch.exp(s - s.amax(-1, keepdim=True))
    o = (p.bfloat16().float() @ v) / p.sum(-1, keepdim=True)
    return o.transpose(1, 2).reshape(B * S, d)


def make_qkv(B, S, heads, seed, scale=1.0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return (torch.randn(B * S, 3 * heads * 64, generator=g, device="cuda") * scale).bfloat16()


@pytest.mark.parametrize("B,S,heads,scale", [(2, 512, 4, 1.0), (1, 128, 2, 1.0), (3, 256, 16, 2.0), (1, 640, 1, 4.0),
                                           (1, 2048, 2, 1.0), (1, 4096, 1, 1.0)])
def test_tcgen05_kernel_vs_reference_and_mma_sync(B, S, heads, scale):
    qkv = make_qkv(B, S, heads, 7 + S, scale)
    ref = reference(qkv, B, S, heads)
    y_tc = attn(qkv, B, S, heads, 0)
    y_mma = attn(qkv, B, S, heads, 1)
    top = ref.abs().max().item()
    assert torch.isfinite(y_tc.float()).all()
    assert (y_tc.float() - ref).abs().max().item() <= TOL * top
    assert (y_mma.float() - ref).abs().max().item() <= TOL * top
    assert (y_tc.float() - y_mma.float()).abs().max().item() <= TOL * top
    assert torch.equal(attn(qkv, B, S, heads, 0), y_tc)


def test_ragged_length_takes_mma_sync_kernel():
    B, S, heads = 2, 200, 2
    qkv = make_qkv(B, S, heads, 3)
    ref = reference(qkv, B, S, heads)
    y = attn(qkv, B, S, heads, 0)
    assert torch.equal(y, attn(qkv, B, S, heads, 1))
    assert (y.float() - ref).abs().max().item() <= TOL * ref.abs().max().item()
