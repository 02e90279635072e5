"""santa_rope_append (LayerCache append, santapp.py:234-274, with the RoPE
of _attention_forward, santapp.py:308-313) is byte work: its rotated queries,
keys and the appended values must equal, bit for bit, what torch computes
from the reference's bf16 expression (transformers' apply_rotary_pos_emb:
q * cos + rotate_half(q) * sin on bf16 tensors) followed by the cache copy,
and the cache outside [start, start + tokens) must stay untouched."""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

from santapp_b200 import _lib  # noqa: E402


def _rotate_half(x):
    x1, x2 = x[..., : x.shape[-1] // 2], x[..., x.shape[-1] // 2:]
    return torch.cat((-x2, x1), dim=-1)


def _rope_cos_sin(B, T, D, start, theta=1e6):
    # Qwen2's rotary embedding: inv_freq over D/2 frequencies, cos/sin of
    # [freqs, freqs] cast to the model dtype
    inv = 1.0 / (theta ** (torch.arange(0, D, 2, dtype=torch.int64).float().cuda() / D))
    pos = torch.arange(start, start + T, device="cuda").float()
    emb = torch.cat([pos[:, None] * inv[None], pos[:, None] * inv[None]], dim=-1)
    cos = emb.cos().to(torch.bfloat16)[None].expand(B, T, D).contiguous()
    sin = emb.sin().to(torch.bfloat16)[None].expand(B, T, D).contiguous()
    return cos, sin


@pytest.mark.parametrize("B,T,Hq,Hkv,D,start,cap", [
    (2, 37, 28, 4, 128, 0, 64),      # prompt into an empty cache
    (3, 1, 28, 4, 128, 511, 520),    # one decode token appended
    (1, 200, 14, 2, 64, 100, 320),   # continued prompt, head_dim 64
])
def test_rope_append_bit_exact(B, T, Hq, Hkv, D, start, cap):
    g = torch.Generator(device="cuda").manual_seed(B * 1000 + T)
    q = (torch.randn(B, T, Hq, D, device="cuda", generator=g) * 3).to(torch.bfloat16)
    k = (torch.randn(B, T, Hkv, D, device="cuda", generator=g) * 3).to(torch.bfloat16)
    v = torch.randn(B, T, Hkv, D, device="cuda", generator=g).to(torch.bfloat16)
    cos, sin = _rope_cos_sin(B, T, D, start)
    kc = torch.randn(B, Hkv, cap, D, device="cuda", generator=g).to(torch.bfloat16)
    vc = torch.randn(B, Hkv, cap, D, device="cuda", generator=g).to(torch.bfloat16)
    kc0, vc0 = kc.clone(), vc.clone()
    q_bf = torch.empty(B, Hq, T, D, dtype=torch.bfloat16, device="cuda")
    q_f32 = torch.empty(B, Hq, T, D, dtype=torch.float32, device="cuda")
    lib = _lib.load()
    _lib.check("santa_rope_append", lib.santa_rope_append(
        B, T, Hq, Hkv, D, q.data_ptr(), k.data_ptr(), v.data_ptr(), cos.data_ptr(),
        sin.data_ptr(), kc.data_ptr(), vc.data_ptr(), cap, start, q_bf.data_ptr(),
        q_f32.data_ptr(), _lib.stream_handle()))
    torch.cuda.synchronize()
    # torch: the reference's expression on [B, H, T, D] bf16 tensors
    qt, kt, vt = q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)
    c, s = cos[:, None], sin[:, None]
    q_ref = (qt * c) + (_rotate_half(qt) * s)
    k_ref = (kt * c) + (_rotate_half(kt) * s)
    assert torch.equal(q_bf, q_ref)
    assert torch.equal(q_f32, q_ref.float())
    assert torch.equal(kc[:, :, start:start + T], k_ref)
    assert torch.equal(vc[:, :, start:start + T], vt)
    # the rest of the cache is untouched
    assert torch.equal(kc[:, :, :start], kc0[:, :, :start])
    assert torch.equal(kc[:, :, start + T:], kc0[:, :, start + T:])
    assert torch.equal(vc[:, :, :start], vc0[:, :, :start])
    assert torch.equal(vc[:, :, start + T:], vc0[:, :, start + T:])


def test_rope_append_rejects_overflow():
    lib = _lib.load()
    x = torch.zeros(16, dtype=torch.bfloat16, device="cuda")
    st = lib.santa_rope_append(1, 4, 1, 1, 2, x.data_ptr(), x.data_ptr(), x.data_ptr(),
                               x.data_ptr(), x.data_ptr(), x.data_ptr(), x.data_ptr(), 4, 1,
                               None, None, _lib.stream_handle())
    assert st == _lib.SANTA_ERR_INVALID_ARGUMENT
