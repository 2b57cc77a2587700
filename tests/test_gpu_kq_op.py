"""GPU counterpart of the reference's ggml fused-KQ op (llama_sp_kq_compute,
src/engine/llama_sp_fused_kq.cpp:82-165) through the C-ABI: scores of one
head's packed rows against every query row, checked against the oracle's
decompressed rows dotted in float64 (float tolerance: 1e-5 relative L2)."""
import ctypes as C

import numpy as np
import pytest

import oracle as O
import spb200
from spb200 import synth

pytestmark = pytest.mark.gpu
KB, VB = [5, 5, 4, 3], [3]


@pytest.mark.parametrize("is_v,n_kv,n_q,qdt", [(0, 1000, 32, "float16"), (1, 257, 5, "float32"),
                                               (0, 4096, 64, "float32"), (0, 1, 1, "float16")])
def test_kq_scores_match_oracle(cuda, is_v, n_kv, n_q, qdt):
    import torch
    L = spb200.lib()
    n = 128
    k, v = synth.kv_slot_np(5, 0, 0, n_kv, n, 1.0)
    rows = O.ship_write(v if is_v else k, VB if is_v else KB, not is_v)     # [n_kv][bytes]
    tb = rows.shape[1]
    packed = torch.from_numpy(rows).cuda()
    q = torch.randn(n_q, n, generator=torch.Generator().manual_seed(n_q)) / 8
    qd = q.to(getattr(torch, qdt)).cuda()
    stride = n_kv + 3                                    # padded dst rows, as ggml's nb[1] may be
    dst = torch.full((n_q, stride), 7.0, dtype=torch.float32, device="cuda")
    rc = L.sp_cuda_kq_scores(packed.data_ptr(), tb, is_v, n, n_kv, qd.data_ptr(),
                             1 if qdt == "float16" else 0, qd.stride(0) * qd.element_size(), n_q,
                             dst.data_ptr(), stride * 4, None)
    assert rc == 0
    torch.cuda.synchronize()
    rec = O.ship_read(rows, n, VB if is_v else KB, not is_v).astype(np.float64)   # [n_kv][n]
    ref = qd.float().cpu().numpy().astype(np.float64) @ rec.T                      # [n_q][n_kv]
    got = dst.cpu().numpy()
    err = np.linalg.norm(got[:, :n_kv] - ref) / max(np.linalg.norm(ref), 1e-30)
    assert err <= 1e-5, err
    assert np.all(got[:, n_kv:] == 7.0)                  # padding untouched


@pytest.mark.parametrize("is_v", [0, 1])
def test_kq_scores_strided_matches_per_slot_calls(cuda, is_v):
    """One launch over several slots (padded slot strides for rows, queries
    and scores) equals one call per slot, bit for bit, and the oracle."""
    import torch
    L = spb200.lib()
    n, n_kv, n_q, n_slots = 128, 777, 4, 5
    tb = 50 if is_v else 76
    max_seq = 800
    slab = torch.zeros(n_slots, max_seq * tb, dtype=torch.uint8)
    recs = []
    for sl in range(n_slots):
        k, v = synth.kv_slot_np(6, 0, sl, n_kv, n, 1.0)
        rows = O.ship_write(v if is_v else k, VB if is_v else KB, not is_v)
        slab[sl, :n_kv * tb] = torch.from_numpy(rows.reshape(-1))
        recs.append(O.ship_read(rows, n, VB if is_v else KB, not is_v).astype(np.float64))
    slab = slab.cuda()
    q = (torch.randn(n_slots, n_q + 1, n, generator=torch.Generator().manual_seed(3)) / 8).half().cuda()
    dst = torch.full((n_slots, n_q, n_kv + 5), 7.0, dtype=torch.float32, device="cuda")
    rc = L.sp_cuda_kq_scores_strided(slab.data_ptr(), max_seq * tb, n_slots, tb, is_v, n, n_kv, q.data_ptr(), 1,
                                     n * 2, (n_q + 1) * n * 2, n_q, dst.data_ptr(), (n_kv + 5) * 4,
                                     n_q * (n_kv + 5) * 4, None)
    assert rc == 0, spb200.last_error()
    one = torch.full_like(dst, 7.0)
    for sl in range(n_slots):
        assert L.sp_cuda_kq_scores(slab[sl].data_ptr(), tb, is_v, n, n_kv, q[sl].data_ptr(), 1, n * 2, n_q,
                                   one[sl].data_ptr(), (n_kv + 5) * 4, None) == 0
    torch.cuda.synchronize()
    assert torch.equal(dst, one)
    got = dst.cpu().numpy()
    for sl in range(n_slots):
        ref = q[sl, :n_q].float().cpu().numpy().astype(np.float64) @ recs[sl].T
        err = np.linalg.norm(got[sl, :, :n_kv] - ref) / np.linalg.norm(ref)
        assert err <= 1e-5, (sl, err)
    assert np.all(got[:, :, n_kv:] == 7.0)


def test_kq_scores_rejects_other_shapes(cuda):
    import torch
    L = spb200.lib()
    buf = torch.zeros(1024, dtype=torch.uint8, device="cuda")
    q = torch.zeros(4, 64, dtype=torch.float16, device="cuda")
    dst = torch.zeros(4, 8, device="cuda")
    assert L.sp_cuda_kq_scores(buf.data_ptr(), 42, 0, 64, 8, q.data_ptr(), 1, 128, 4, dst.data_ptr(), 32,
                               None) == spb200.SP_ERR_UNSUPPORTED
