"""The attention entry point that allocates nothing.

Callers that cannot call cudaMalloc while serving (a host that owns a fixed
device arena, or a plugin that is only handed input and output pointers) use
af_attention_decode_f32_noalloc, whose scratch is a fixed array inside the
library.  Its output must match af_attention_decode_f32 with caller-provided
scratch, on two calls in a row (the shared scratch keeps the previous call's
contents).  This file is collected last on purpose."""
import numpy as np
import pytest

from helpers import dev, rel_l2
from oracle import COracle

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("H,KVH,hd,pos,nsplit", [(32, 32, 128, 200, 10), (16, 2, 128, 1000, 64), (32, 4, 64, 77, 37)])
def test_noalloc_attention_matches_scratch_version(gpu, H, KVH, hd, pos, nsplit):
    import torch
    rng = np.random.default_rng(H * 7 + pos)
    n_ctx = 2048
    kvd = KVH * hd
    c, s = COracle().rope_tables(hd, 10000.0, n_ctx)
    kc = np.zeros((n_ctx, kvd), np.float32)
    vc = np.zeros((n_ctx, kvd), np.float32)
    kc[:pos + 2] = rng.standard_normal((pos + 2, kvd))
    vc[:pos + 2] = rng.standard_normal((pos + 2, kvd))
    cd, sd = dev(c), dev(s)
    part = torch.zeros(H * nsplit * (hd + 2), device="cuda")
    cnt = torch.zeros(KVH, dtype=torch.int32, device="cuda")
    for call in range(2):  # two calls in a row, at consecutive positions
        p = pos + call
        q = rng.standard_normal(H * hd).astype(np.float32)
        k = rng.standard_normal(kvd).astype(np.float32)
        v = rng.standard_normal(kvd).astype(np.float32)
        qd, kd, vd = dev(q), dev(k), dev(v)
        posd = torch.tensor([p], dtype=torch.int32, device="cuda")
        outs = []
        for noalloc in (False, True):
            kcd, vcd = dev(kc), dev(vc)
            out = torch.full((H * hd,), float("nan"), device="cuda")
            args = [out.data_ptr(), qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), kcd.data_ptr(), vcd.data_ptr(),
                    cd.data_ptr(), sd.data_ptr(), None, None, posd.data_ptr(), H, KVH, hd, n_ctx, 0, 1e-5, nsplit]
            if noalloc:
                rc = gpu.af_attention_decode_f32_noalloc(*args, None)
            else:
                rc = gpu.af_attention_decode_f32(*args, part.data_ptr(), cnt.data_ptr(), None)
            assert rc == 0, gpu.af_last_error()
            torch.cuda.synchronize()
            outs.append((out.cpu().numpy(), kcd.cpu().numpy()[p], vcd.cpu().numpy()[p]))
        (o_ref, k_ref, v_ref), (o_na, k_na, v_na) = outs
        assert np.isfinite(o_na).all()
        assert rel_l2(o_na, o_ref) < 1e-5
        assert np.array_equal(k_na, k_ref) and np.array_equal(v_na, v_ref)


def test_noalloc_rejects_oversized_calls(gpu):
    # 64 heads * 64 splits * 130 floats > the fixed 262144-float scratch
    rc = gpu.af_attention_decode_f32_noalloc(None, None, None, None, None, None, None, None, None, None, None,
                                             64, 64, 128, 4096, 0, 1e-5, 64, None)
    assert rc != 0
    assert b"262144" in gpu.af_last_error()
