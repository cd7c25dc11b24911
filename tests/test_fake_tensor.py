"""Every attnres:: operator has a fake (meta) implementation, so graphs that
contain it can be traced (torch.compile / export) without running CUDA: the
reference registers its ops for the same reason (attnres_ops.py:4632)."""
import torch
from torch._subclasses.fake_tensor import FakeTensorMode

import attnres_b200  # noqa: F401  (registers torch.ops.attnres.*)


def _fake(mode, *shape, dtype=torch.bfloat16):
    with mode:
        return torch.empty(*shape, dtype=dtype, device="cuda")


def test_fake_shapes_of_all_ops():
    mode = FakeTensorMode(allow_non_fake_inputs=False)
    S, B, T, D, R, H, Q = 5, 2, 7, 64, 16, 2, 3
    v = [_fake(mode, B, T, D) for _ in range(S)]
    k = [_fake(mode, B, T, R) for _ in range(S)]
    q = _fake(mode, H, R // H)
    g = _fake(mode, B, T, D)
    ops = torch.ops.attnres
    with mode:
        out, inv, alpha, kinv = ops.lrid_read_list(v, k, q, H, 0.5, True, False, True)
        assert out.shape == (B, T, D) and alpha.shape == (B * T, H, S)
        gv, gk, dq = ops.lrid_read_list_backward(v, k, q, g, out, inv, alpha, kinv, H, 0.5, True, False, True)
        assert len(gv) == S and gk[0].shape == (B, T, R) and dq.shape == q.shape
        out2, inv2 = ops.lrid_read(v, k, q, None, None, None, H, 0.5, True, 2)
        assert inv2.shape == (B * T,)
        w = _fake(mode, R, D)
        o, oi, keys, vinv, al = ops.lrid_kv_read(v, w, q, None, None, None, H, 0.5, True, 0, True)
        assert keys.shape == (S, B, T, R) and vinv.shape == (S, B * T) and al.shape == (B * T, H, S)
        lg = _fake(mode, Q, S, B, T, dtype=torch.float32)
        po, lse, pinv = ops.phase1_from_logits(v, lg, False)
        assert po.shape == (Q, B, T, D) and lse.shape == (Q, B, T)
        bo, binv = ops.base_read(v, _fake(mode, D), None, True, True)
        assert bo.shape == (B, T, D) and binv.shape == (B * T,)
        fo, fk, fq, fi = ops.lrid_fused_projection(v[0], _fake(mode, D + R + R, D), D, R, H, True, R)
        assert fo.shape == (B, T, D) and fk.shape == (B, T, R) and fq.shape == (B, T, R) and fi.shape == (B * T, H)
        ssum, ssrc = ops.block_summary(v[0], v[1], None, 0.5)
        assert ssum.shape == (B, T, D) and ssrc.shape == (B, T, D)
        p2o, p2i = ops.phase2(0, v[0], k[0], None, _fake(mode, R), v[1], _fake(mode, B, T, dtype=torch.float32),
                              0.5, True, None, 0.0, True)
        assert p2o.shape == (B, T, D) and p2i.shape == (B * T,)
        p2g = ops.phase2_backward(0, v[0], k[0], None, _fake(mode, R), v[1], _fake(mode, B, T, dtype=torch.float32),
                                  0.5, True, None, 0.0, True, p2o, p2i, g, True, False)
        assert p2g[0].shape == (B * T, D) and p2g[1].shape == (B * T, R) and p2g[5].shape == (R,)
        gp, gsc = ops.block_summary_backward(g, None, ssum, _fake(mode, 1, dtype=torch.float32), 1.0, True)
        assert gp.shape == (B, T, D) and gsc.shape == (1,)
