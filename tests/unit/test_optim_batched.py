"""Batched NorMuon (one Polar-Express chain per shape group) against the per-matrix update."""

import torch

from mint_b200.optim.functional import normuon_update, normuon_update_batched, polar_express, polar_express_batched


def test_polar_express_batched_matches_per_matrix():
    torch.manual_seed(0)
    for shape in ((3, 32, 16), (2, 16, 48), (4, 24, 24)):
        g = torch.randn(*shape)
        got = polar_express_batched(g, 5)
        for i in range(shape[0]):
            torch.testing.assert_close(got[i], polar_express(g[i], 5), rtol=1e-4, atol=1e-5)


def test_normuon_batched_matches_per_matrix():
    torch.manual_seed(1)
    n, rows, cols = 3, 40, 24
    params = [torch.randn(rows, cols) for _ in range(n)]
    ref_params = [p.clone() for p in params]
    mb = torch.zeros(n, rows, cols)
    smb = torch.zeros(n, rows, 1)
    ref_state = [(torch.zeros(rows, cols), torch.zeros(rows, 1)) for _ in range(n)]
    kw = dict(lr=0.02, momentum=0.95, beta2=0.95, wd=0.1, ns_steps=5)
    for _step in range(3):
        grads = torch.randn(n, rows, cols)
        normuon_update_batched(params, grads, mb, smb, **kw)
        for i in range(n):
            normuon_update(ref_params[i], grads[i].clone(), ref_state[i][0], ref_state[i][1], **kw)
    for i in range(n):
        torch.testing.assert_close(params[i], ref_params[i], rtol=1e-4, atol=1e-5)
        torch.testing.assert_close(mb[i], ref_state[i][0], rtol=1e-5, atol=1e-6)
        torch.testing.assert_close(smb[i], ref_state[i][1], rtol=1e-4, atol=1e-6)
