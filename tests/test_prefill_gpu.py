"""GPU parity of the tcgen05 prefill (causal / non-causal / var-len) against the
CPU oracle and the reference's golden outputs.

Tolerance: max-abs <= 2e-3 against the fp32 oracle, no NaNs (bf16 adds half a
bf16 ulp of the reference value, and where many rows are checked in bf16 also
2^-9 * max|V| for the bf16 rounding of P before P.V).  The kernel rounds P to the input dtype
before P.V, as the reference does (PF:94); the oracle keeps P in fp32.
"""
import math

import pytest
import torch

from golden_io import load
from oracle import naive as N

from attention_kernel_triton_b200 import _lib
from attention_kernel_triton_b200 import workloads as W
from attention_kernel_triton_b200.prefill_flash_attention import flash_attention_prefill
from attention_kernel_triton_b200.prefill_flash_attention_var_len_padding import (
    flash_attention_prefill as flash_attention_prefill_varlen)

pytestmark = pytest.mark.gpu
TOL = 2e-3
DEV = "cuda"


def check_close(out, ref, dtype=torch.float16, extra=0.0):
    out = out.detach().float().cpu()
    ref = ref.detach().float().cpu()
    assert out.shape == ref.shape
    assert not torch.isnan(out).any()
    err = (out - ref).abs()
    bound = TOL + extra + (2.0 ** -8 * ref.abs() if dtype == torch.bfloat16 else 0.0)
    assert bool((err <= bound).all()), f"max err {err.max().item()} at {divmod(int(err.argmax()), out.shape[-1])}"


@pytest.fixture(autouse=True)
def device_status_clean():
    _lib.device_status(0, clear=True)
    yield
    assert _lib.device_status(0) == 0, "a kernel recorded an error"


def cuda(x):
    return x.to(DEV)


@pytest.mark.parametrize("name", ["prefill_causal_gqa", "prefill_noncausal", "prefill_causal_d128"])
def test_prefill_matches_reference_golden(name):
    f = load(name)
    O = flash_attention_prefill(cuda(f["Q"]), cuda(f["K"]), cuda(f["V"]), f["causal"], f["softmax_scale"], f["group"])
    assert O.shape == f["O"].shape and O.dtype == torch.float16
    check_close(O, f["O"])
    check_close(O, N.prefill_reference(f["Q"], f["K"], f["V"], f["causal"], f["softmax_scale"], f["group"]))


def test_prefill_varlen_matches_reference_golden():
    f = load("prefill_varlen")
    O = flash_attention_prefill_varlen(cuda(f["Q"]), cuda(f["K"]), cuda(f["V"]), True, f["softmax_scale"],
                                       f["group"], cuda(f["varlen"]))
    check_close(O, f["O"])


@pytest.mark.parametrize("causal", [True, False])
@pytest.mark.parametrize("S", [1, 64, 100, 128, 129, 300])
@pytest.mark.parametrize("D,G", [(64, 1), (64, 4), (128, 2), (128, 8)])
def test_prefill_shapes(causal, S, D, G):
    c = W.make_prefill(B=2, Hq=2 * G, Hkv=2, S=S, D=D, causal=causal, seed=S * 10 + D + G)
    O = flash_attention_prefill(cuda(c.Q), cuda(c.K), cuda(c.V), causal, c.softmax_scale, G)
    check_close(O, N.prefill_reference(c.Q, c.K, c.V, causal, c.softmax_scale, G))


@pytest.mark.parametrize("D", [64, 128])
def test_prefill_bf16(D):
    c = W.make_prefill(B=1, Hq=4, Hkv=1, S=257, D=D, causal=True, seed=5, dtype=torch.bfloat16)
    O = flash_attention_prefill(cuda(c.Q), cuda(c.K), cuda(c.V), True, c.softmax_scale, 4)
    assert O.dtype == torch.bfloat16
    check_close(O, N.prefill_reference(c.Q, c.K, c.V, True, c.softmax_scale, 4), torch.bfloat16)


def test_causal_row_zero_is_v_row_zero_exactly():
    c = W.make_prefill(B=2, Hq=8, Hkv=2, S=200, D=64, causal=True, seed=6)
    O = flash_attention_prefill(cuda(c.Q), cuda(c.K), cuda(c.V), True, c.softmax_scale, 4)
    Vx = c.V.repeat_interleave(4, dim=1)
    assert torch.equal(O[:, :, 0].cpu(), Vx[:, :, 0])


@pytest.mark.parametrize("causal", [True, False])
def test_prefill_varlen_shapes(causal):
    c = W.make_prefill(B=4, Hq=8, Hkv=2, S=384, D=64, causal=causal, seed=7)
    lens = torch.tensor([384, 1, 129, 200], dtype=torch.int64)  # reference passes an int64 tensor
    O = flash_attention_prefill_varlen(cuda(c.Q), cuda(c.K), cuda(c.V), causal, c.softmax_scale, 4, cuda(lens))
    check_close(O, N.prefill_varlen_reference(c.Q, c.K, c.V, causal, c.softmax_scale, 4, lens))


# The var-len kernel orders its work from the lengths (real query tiles by
# causal cost, then the tiles past each sequence's length); these cases cover
# zero-length and one-row sequences, ties, D=128, odd groups and plain
# multi-head attention (one query head and two query tiles per item) and more
# batches than the order table holds (plain order).  Output is independent of the order, so all match the oracle.
@pytest.mark.parametrize("B,Hq,Hkv,S,D,lens", [
    (6, 8, 2, 384, 64, [0, 384, 5, 384, 250, 128]),
    (5, 8, 2, 300, 128, [300, 0, 77, 299, 1]),
    (4, 6, 2, 256, 64, [256, 0, 129, 40]),
    (5, 4, 4, 640, 64, [640, 3, 0, 257, 600]),
    (3, 3, 3, 300, 128, [1, 300, 130]),
    (257, 2, 1, 64, 64, None),
])
def test_prefill_varlen_work_order(B, Hq, Hkv, S, D, lens):
    c = W.make_prefill(B=B, Hq=Hq, Hkv=Hkv, S=S, D=D, causal=True, seed=21)
    if lens is None:
        g = torch.Generator().manual_seed(22)
        lens = torch.randint(0, S + 1, (B,), generator=g, dtype=torch.int64).tolist()
    lens = torch.tensor(lens, dtype=torch.int32)
    G = Hq // Hkv
    O = flash_attention_prefill_varlen(cuda(c.Q), cuda(c.K), cuda(c.V), True, c.softmax_scale, G, cuda(lens))
    check_close(O, N.prefill_varlen_reference(c.Q, c.K, c.V, True, c.softmax_scale, G, lens))


def test_prefill_strided_inputs():
    c = W.make_prefill(B=2, Hq=4, Hkv=2, S=150, D=64, causal=True, seed=8)
    Qt = cuda(c.Q).transpose(1, 2).contiguous().transpose(1, 2)   # [B,H,S,D] view, token-major storage
    Kt = cuda(c.K).transpose(1, 2).contiguous().transpose(1, 2)
    O = flash_attention_prefill(Qt, Kt, cuda(c.V), True, c.softmax_scale, 2)
    check_close(O, N.prefill_reference(c.Q, c.K, c.V, True, c.softmax_scale, 2))


def test_prefill_reference_asserts():
    Q = torch.zeros(1, 4, 64, 96, dtype=torch.float16, device=DEV)
    with pytest.raises(AssertionError):
        flash_attention_prefill(Q, Q[:, :2], Q[:, :2], True, 0.1, 2)
    with pytest.raises(AssertionError):
        flash_attention_prefill(Q[..., :64], Q[:, :1, :, :64], Q[:, :1, :, :64], True, 0.1, 2)


# ---------------------------------------------------------------- cfg0 / cfg1 (B=8, Hq=64, Hkv=16, S=1024, D=64), full size
def _sampled_ref(c, heads, varlen=None):
    B, H, S, D = c.Q.shape
    out = {}
    for (b, h) in heads:
        kvh = h // c.group
        Q = c.Q[b:b + 1, h:h + 1].cpu()
        K = c.K[b:b + 1, kvh:kvh + 1].cpu()
        V = c.V[b:b + 1, kvh:kvh + 1].cpu()
        if varlen is None:
            out[(b, h)] = N.prefill_reference(Q, K, V, c.causal, c.softmax_scale, 1)[0, 0]
        else:
            out[(b, h)] = N.prefill_varlen_reference(Q, K, V, c.causal, c.softmax_scale, 1, varlen[b:b + 1])[0, 0]
    return out


def test_prefill_cfg0_full_size_sampled():
    c = W.make_prefill(seed=0, device=DEV)  # Q [8,64,1024,64], K/V [8,16,1024,64], causal, fp16
    O = flash_attention_prefill(c.Q, c.K, c.V, True, c.softmax_scale, c.group)
    assert O.shape == (8, 64, 1024, 64) and not torch.isnan(O).any()
    heads = [(0, 0), (3, 17), (7, 63), (5, 40)]
    for k, ref in _sampled_ref(c, heads).items():
        check_close(O[k[0], k[1]], ref)


def test_prefill_cfg1_varlen_full_size_sampled():
    c = W.make_prefill(seed=1, device=DEV, varlen=True)
    O = flash_attention_prefill_varlen(c.Q, c.K, c.V, True, c.softmax_scale, c.group, c.varlen)
    lens = c.varlen.cpu()
    heads = [(0, 5), (1, 33), (int(lens.argmin()), 7), (6, 62)]
    for k, ref in _sampled_ref(c, heads, lens).items():
        check_close(O[k[0], k[1]], ref)
    for b in range(8):
        assert torch.all(O[b, :, int(lens[b]):] == 0)


# ---------------------------------------------------------------- LSE output (PF:331-334, unstored there)
LSE_TOL = 1e-3  # fp32 log-sum-exp of fp32-accumulated scores; exp2 approximations in the kernel


@pytest.mark.parametrize("causal", [True, False])
@pytest.mark.parametrize("S,D,G", [(1, 64, 1), (129, 64, 4), (300, 128, 2), (256, 64, 2)])
def test_prefill_lse_matches_oracle(causal, S, D, G):
    from attention_kernel_triton_b200.prefill_flash_attention import flash_attention_prefill_with_lse
    c = W.make_prefill(B=2, Hq=2 * G, Hkv=2, S=S, D=D, causal=causal, seed=S + D + G)
    O, LSE = flash_attention_prefill_with_lse(cuda(c.Q), cuda(c.K), cuda(c.V), causal, c.softmax_scale, G)
    O_plain = flash_attention_prefill(cuda(c.Q), cuda(c.K), cuda(c.V), causal, c.softmax_scale, G)
    assert torch.equal(O, O_plain)
    ref = N.prefill_lse_reference(c.Q, c.K, c.V, causal, c.softmax_scale, G)
    assert LSE.shape == ref.shape and LSE.dtype == torch.float32
    assert (LSE.cpu() - ref).abs().max().item() <= LSE_TOL


@pytest.mark.parametrize("Hq,Hkv,dtype", [(4, 4, torch.float16), (8, 2, torch.bfloat16), (3, 1, torch.bfloat16)])
def test_prefill_varlen_lse_ordered_variants(Hq, Hkv, dtype):
    """The var-len kernels that order their work from the lengths, with the LSE
    output: multi-head (one head, two query tiles per item), bf16 with an even
    and an odd group; zero-length and one-row sequences included."""
    from attention_kernel_triton_b200.prefill_flash_attention_var_len_padding import flash_attention_prefill_with_lse
    c = W.make_prefill(B=4, Hq=Hq, Hkv=Hkv, S=333, D=64, causal=True, seed=31, dtype=dtype)
    lens = torch.tensor([333, 0, 1, 200], dtype=torch.int32)
    G = Hq // Hkv
    O, LSE = flash_attention_prefill_with_lse(cuda(c.Q), cuda(c.K), cuda(c.V), True, c.softmax_scale, G, cuda(lens))
    assert O.dtype == dtype
    ref = N.prefill_lse_reference(c.Q, c.K, c.V, True, c.softmax_scale, G, lens)
    fin = torch.isfinite(ref)
    assert torch.equal(torch.isfinite(LSE.cpu()), fin)
    assert (LSE.cpu()[fin] - ref[fin]).abs().max().item() <= LSE_TOL
    # bf16: P is rounded to bf16 before P.V, as in the reference (PF:94), so each
    # weight carries up to 2^-9 relative error and O may move by 2^-9 * max|V|
    # against the fp32 oracle, beyond the output's own rounding
    extra = 2.0 ** -9 * c.V.float().abs().max().item() if dtype == torch.bfloat16 else 0.0
    check_close(O, N.prefill_varlen_reference(c.Q, c.K, c.V, True, c.softmax_scale, G, lens), dtype, extra)


def test_prefill_varlen_lse_padding_rows_are_minus_inf():
    from attention_kernel_triton_b200.prefill_flash_attention_var_len_padding import flash_attention_prefill_with_lse
    c = W.make_prefill(B=3, Hq=8, Hkv=2, S=300, D=64, causal=True, seed=9)
    lens = torch.tensor([300, 1, 130], dtype=torch.int32)
    O, LSE = flash_attention_prefill_with_lse(cuda(c.Q), cuda(c.K), cuda(c.V), True, c.softmax_scale, 4, cuda(lens))
    ref = N.prefill_lse_reference(c.Q, c.K, c.V, True, c.softmax_scale, 4, lens)
    fin = torch.isfinite(ref)
    assert torch.equal(torch.isfinite(LSE.cpu()), fin)
    assert (LSE.cpu()[fin] - ref[fin]).abs().max().item() <= LSE_TOL
    check_close(O, N.prefill_varlen_reference(c.Q, c.K, c.V, True, c.softmax_scale, 4, lens))


def test_prefill_lse_merges_two_key_halves_like_split_kv():
    # LSE is what lets partial outputs over disjoint key sets be merged: a non-causal
    # prefill over keys [0, S/2) and [S/2, S) merged with akt_lse_merge equals the full one
    from attention_kernel_triton_b200.distributed import lse_merge_into
    from attention_kernel_triton_b200.prefill_flash_attention import flash_attention_prefill_with_lse
    c = W.make_prefill(B=1, Hq=4, Hkv=4, S=256, D=64, causal=False, seed=10)
    Q, K, V = cuda(c.Q), cuda(c.K), cuda(c.V)
    parts = []
    for lo, hi in [(0, 128), (128, 256)]:  # the first 128 queries against each half of the keys
        O_h, L_h = flash_attention_prefill_with_lse(Q[:, :, :128], K[:, :, lo:hi], V[:, :, lo:hi], False,
                                                    c.softmax_scale, 1)
        parts.append((O_h.float(), L_h))
    rows, D = 4 * 128, 64
    recv = torch.cat([torch.cat([o.reshape(1, -1), l.reshape(1, -1)], dim=1) for o, l in parts], dim=0)
    out = torch.empty(rows, D, dtype=torch.float16, device=DEV)
    lse_merge_into(out, recv, rows, D)
    full = N.prefill_reference(c.Q[:, :, :128], c.K, c.V, False, c.softmax_scale, 1)
    check_close(out.reshape(1, 4, 128, 64), full)
