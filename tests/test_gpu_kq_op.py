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


def test_kq_scores_rejects_other_shapes(cuda):
    import torch
    L = spb200.lib()
    buf = torch.zeros(1024, dtype=torch.uint8, device="cuda")
    q = torch.zeros(4, 64, dtype=torch.float16, device="cuda")
    dst = torch.zeros(4, 8, device="cuda")
    assert L.sp_cuda_kq_scores(buf.data_ptr(), 42, 0, 64, 8, q.data_ptr(), 1, 128, 4, dst.data_ptr(), 32,
                               None) == spb200.SP_ERR_UNSUPPORTED
