"""SageAttention over the FP8 cache on the B200 kernels against the CPU oracle (oracle/sage.py): the quantized
operands in value space (Q INT8 and scales bitwise; K INT8 within +-1 and its scales to 1e-5, since the key
mean is a float sum in another order; V FP8 bytes >= 99.9 % equal), and the attention output against exact
attention over the cache's values (cosine >= 0.999, the stated bar; the reference's test_sage_kv.py:86-98
style), against the emulation of its own P V over the cache's per-token V (relative L2 < 5e-3), and against the
reference's own Sage arithmetic (V re-quantized per channel) through the exact result: no less accurate than it
within 10 %. Its cosine against the reference's quantized operands is printed: two approximations of the same
result differ from each other by more than either differs from it."""

import numpy as np
import pytest
import torch

from oracle import fp8 as of
from oracle import sage as osage

pytestmark = pytest.mark.gpu


def setup(at, n, nq, H, seed=0, k_dtype=torch.float32):
    g = torch.Generator().manual_seed(seed)
    total = at + n + 64
    ck, cks = of.quantize_rows((torch.randn(1, total, H, 128, generator=g) + 0.5).numpy())
    cv, cvs = of.quantize_rows((torch.randn(1, total, H, 128, generator=g) * 0.7).numpy())
    K = (torch.randn(1, n, H, 128, generator=g) + 0.5).to(k_dtype)
    V = torch.randn(1, n, H, 128, generator=g).to(torch.bfloat16)
    Q = torch.randn(1, nq, H, 128, generator=g)
    host = dict(ck=ck, cks=cks, cv=cv, cvs=cvs, K=K.float().numpy(), V=V.float().numpy(), Q=Q.numpy())
    dev = dict(ck=torch.from_numpy(ck).view(torch.float8_e4m3fn).cuda(), cks=torch.from_numpy(cks).cuda(),
               cv=torch.from_numpy(cv).view(torch.float8_e4m3fn).cuda(), cvs=torch.from_numpy(cvs).cuda(),
               K=K.cuda(), V=V.cuda(), Q=Q.cuda())
    return host, dev


def cosine(a, b):
    a, b = np.asarray(a, np.float64).ravel(), np.asarray(b, np.float64).ravel()
    return float(a @ b / np.linalg.norm(a) / np.linalg.norm(b))


@pytest.mark.parametrize("at,n,nq,H", [(200, 150, 150, 2), (0, 300, 300, 1), (4176, 1392, 1392, 24)])
def test_quantized_operands_match_oracle(at, n, nq, H):
    from wan_dit_lab_b200.kernels import sage_kv
    host, d = setup(at, n, nq, H)
    ops = {k: v.cpu().numpy() for k, v in sage_kv.prepare(d["Q"], d["ck"], d["cks"], d["cv"], d["cvs"], at, d["K"],
                                                          d["V"]).items()}
    L = at + n
    Kf = osage.load(host["ck"], host["cks"], host["K"], at)
    Vf = osage.load(host["cv"], host["cvs"], host["V"], at)
    kq, ks, _ = osage.quant_k(Kf)
    qq, qs = osage.quant_q(host["Q"])
    v8, vs = osage.quant_v(Vf)
    # Q: [H, npad, 128] -> [1, nq, H, 128]
    np.testing.assert_array_equal(ops["q_i8"][:, :nq].transpose(1, 0, 2)[None], qq)
    np.testing.assert_array_equal(ops["q_scale"][:, :qs.shape[-1]][None], qs)
    got_k = ops["k_i8"][:, :L].transpose(1, 0, 2)[None].astype(int)
    assert np.abs(got_k - kq.astype(int)).max() <= 1
    assert (got_k == kq).mean() > 0.999
    np.testing.assert_allclose(ops["k_scale"][:, :ks.shape[-1]][None], ks, rtol=1e-5)
    np.testing.assert_allclose(ops["v_scale"][None], vs, rtol=1e-6)
    got_v = ops["v_f8"][:, :, :L].transpose(2, 0, 1)[None]  # [1, L, H, 128]
    assert (got_v == osage.unpermute_v(v8, L)).mean() > 0.999
    assert not ops["k_i8"][:, L:].any() and not ops["v_f8"][:, :, L:].any()  # zero padding


@pytest.mark.parametrize("at,n,nq,H", [(200, 150, 150, 2), (0, 300, 300, 1), (4176, 1392, 1392, 24), (9360, 3120, 3120, 2),
                                        (15840, 2640, 2640, 1)])  # config 5: 18480 keys, 145 key tiles
def test_attention_matches_oracle(at, n, nq, H):
    from wan_dit_lab_b200.kernels import sage_kv
    from wan_dit_lab_b200 import _native
    host, d = setup(at, n, nq, H, seed=at + n)
    out = sage_kv.attend(d["Q"], d["ck"], d["cks"], d["cv"], d["cvs"], at, d["K"], d["V"]).float().cpu().numpy()
    assert _native.device_error() == 0
    quantized = osage.sage_attention(host["Q"], host["ck"], host["cks"], host["cv"], host["cvs"], at, host["K"], host["V"])
    exact = osage.attention(host["Q"], osage.load(host["ck"], host["cks"], host["K"], at),
                            osage.load(host["cv"], host["cvs"], host["V"], at))
    emulated = osage.sage_attention(host["Q"], host["ck"], host["cks"], host["cv"], host["cvs"], at, host["K"], host["V"],
                                    fp8_p=True, token_v=True)
    assert float(np.linalg.norm(out - emulated) / np.linalg.norm(emulated)) < 5e-3  # the kernel's own FP8 P V
    reference = osage.sage_attention(host["Q"], host["ck"], host["cks"], host["cv"], host["cvs"], at, host["K"],
                                     host["V"], fp8_p=True)  # the reference's P V: V re-quantized per channel
    c_q, c_e = cosine(out, quantized), cosine(out, exact)
    err = lambda x: float(np.linalg.norm(x - exact) / np.linalg.norm(exact))  # noqa: E731
    print(f"at {at} n {n}: cos vs dequantized {c_q:.6f}, vs exact {c_e:.6f}; rel err kernel {err(out):.4f}, "
          f"the reference's Sage arithmetic {err(reference):.4f}, dequantized oracle {err(quantized):.4f}")
    assert c_e >= 0.999  # the stated bar, against attention over the cache's values
    assert err(out) < 1.2 * err(quantized) + 2e-2  # P in FP8 adds its own rounding on top of Q / K / V's
    # no less accurate than the reference's own arithmetic (two approximations differ from each other by more
    # than either does from the exact result, so they are compared through it)
    assert err(out) <= 1.1 * err(reference)


def test_attend_rejects_invalid_contracts():
    from wan_dit_lab_b200.kernels import sage_kv
    host, d = setup(20, 10, 10, 1)
    with pytest.raises(ValueError):
        sage_kv.attend(d["Q"], d["ck"], d["cks"], d["cv"], d["cvs"], 10 ** 6, d["K"], d["V"])
    with pytest.raises(ValueError):  # a head map must be int32 [H]
        sage_kv.attend(d["Q"], d["ck"], d["cks"], d["cv"], d["cvs"], 20, d["K"], d["V"], heads=torch.zeros(1))
    with pytest.raises(TypeError):
        sage_kv.attend(d["Q"], d["ck"].float(), d["cks"], d["cv"], d["cvs"], 20, d["K"], d["V"])


@pytest.mark.parametrize("at,n,H,cache_heads", [(200, 150, 2, 4), (1392, 1392, 3, 8)])
def test_forcing_kv_maps_equal_a_gathered_cache(at, n, H, cache_heads):
    """Head and token maps (Forcing-KV, sage_kv.py:127-134) read the cache in place: the result equals, bit for bit,
    attention over a copy of the cache gathered through the same maps."""
    from wan_dit_lab_b200.kernels import sage_kv
    from wan_dit_lab_b200 import _native
    rows = at + 300
    _, d = setup(rows, n, n, cache_heads, seed=7)
    g = torch.Generator().manual_seed(8)
    heads = torch.randperm(cache_heads, generator=g)[:H].to(torch.int32).cuda()
    tokens = torch.randperm(rows, generator=g)[:at].to(torch.int32).cuda()
    Q, K, V = (d[x][:, :, :H].contiguous() for x in ("Q", "K", "V"))
    got = sage_kv.attend(Q, d["ck"], d["cks"], d["cv"], d["cvs"], at, K, V, heads=heads, tokens=tokens)
    assert _native.device_error() == 0
    t, h = tokens.long(), heads.long()
    gather = lambda c: c[:, t][:, :, h].contiguous()  # noqa: E731
    want = sage_kv.attend(Q, gather(d["ck"]), gather(d["cks"]), gather(d["cv"]), gather(d["cvs"]), at, K, V)
    torch.cuda.synchronize()
    assert torch.equal(got, want)
    # heads alone over the whole window, tokens alone with every head
    got_h = sage_kv.attend(Q, d["ck"], d["cks"], d["cv"], d["cvs"], at, K, V, heads=heads)
    want_h = sage_kv.attend(Q, d["ck"][:, :, h].contiguous(), d["cks"][:, :, h].contiguous(),
                            d["cv"][:, :, h].contiguous(), d["cvs"][:, :, h].contiguous(), at, K, V)
    assert torch.equal(got_h, want_h)
    assert _native.device_error() == 0


def test_forcing_kv_map_out_of_range_is_reported():
    """A token map entry past the cache is caught by the kernel's own bounds check: read as row 0, reported."""
    from wan_dit_lab_b200.kernels import sage_kv
    from wan_dit_lab_b200 import _native
    at, n, H = 64, 64, 1
    _, d = setup(at, n, n, H, seed=9)
    tokens = torch.arange(at, dtype=torch.int32).cuda()
    tokens[5] = d["ck"].shape[1] + 1000
    out = sage_kv.attend(d["Q"], d["ck"], d["cks"], d["cv"], d["cvs"], at, d["K"], d["V"], tokens=tokens)
    with pytest.raises(RuntimeError, match="index map.*code 7"):
        _native.device_error()
    assert torch.isfinite(out.float()).all()
    assert _native.device_error() == 0  # read and cleared


@pytest.mark.parametrize("at,n,H", [(200, 150, 2), (256, 100, 1), (0, 300, 2), (4176, 1392, 3)])
def test_values_stored_in_the_cache_equal_values_given(at, n, H):
    """P V reads V as the cache holds it. The chunk's values passed in 16 bits (quantized by the call into its
    workspace, the keys before `at` of their 128-key tile copied beside them) and the same values stored in the
    cache first by the cache's own store (cache_fp8.store_kv_fp8) and read from there (v null, as the model calls
    it after wdl_qkv_prep) give the same attention, bit for bit."""
    from wan_dit_lab_b200 import _native
    from wan_dit_lab_b200.kernels import cache_fp8, sage_kv
    _, d = setup(at, n, n, H, seed=11 + at)
    given = sage_kv.attend(d["Q"], d["ck"], d["cks"], d["cv"], d["cvs"], at, d["K"], d["V"])
    ck, cks, cv, cvs = (d[x].clone() for x in ("ck", "cks", "cv", "cvs"))
    cache_fp8.store_kv_fp8(d["K"], d["V"], ck, cks, cv, cvs, at)
    lib = _native.lib()
    L = at + n
    q = d["Q"][0].reshape(n, H * 128).contiguous()
    k = d["K"][0].reshape(n, H * 128).contiguous()
    out = torch.empty(n, H * 128, dtype=torch.bfloat16, device="cuda")
    work = torch.empty(lib.wdl_sage_attend_workspace(n, L, H), dtype=torch.uint8, device="cuda")
    _native.check(lib.wdl_sage_attend(q.data_ptr(), H * 128, n, ck.data_ptr(), cks.data_ptr(), cv.data_ptr(),
                                      cvs.data_ptr(), at, k.data_ptr(), _native.F32, H * 128, None, _native.BF16,
                                      H * 128, n, H, 128 ** -0.5, out.data_ptr(), H * 128, work.data_ptr(),
                                      work.numel(), _native.stream()))
    torch.cuda.synchronize()
    assert _native.device_error() == 0
    assert torch.equal(out, given[0].reshape(n, H * 128))
    # with index maps the chunk's values are required
    st = lib.wdl_sage_attend_maps(q.data_ptr(), H * 128, n, ck.data_ptr(), cks.data_ptr(), cv.data_ptr(),
                                  cvs.data_ptr(), ck.shape[1], H, None, None, at, k.data_ptr(), _native.F32, H * 128,
                                  None, _native.BF16, H * 128, n, H, 128 ** -0.5, out.data_ptr(), H * 128,
                                  work.data_ptr(), work.numel(), _native.stream())
    assert st == _native.ERR_ARGUMENT
