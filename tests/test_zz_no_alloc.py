"""trc_moe_couche_sans_alloc: the fused layer on the library's fixed device workspace.

- on the GPU, through the C-ABI: two calls in a row (different inputs, one stream, no
  synchronisation between them) give the bits of trc_moe_couche_fusionnee with a workspace of
  the caller's own on the same inputs (tolerance zero: the same kernels on the same inputs),
  for a small layer and the gpt-oss-120b shapes at k = 4 and k = 8 (6,865,920 of the 8 MiB);
- without a GPU: a layer whose workspace would exceed the fixed 8 MiB is refused with a usage
  error before anything is launched, and so is a missing descriptor.

This file is collected last so that it runs both after the other tests and, alone, in a fresh
process."""
import ctypes as C

import numpy as np
import pytest

import troncons_b200 as T

LIMITE = 8 << 20


def test_refuse_au_dela_de_la_limite():
    dims = T.DimsExpert.de([8192, 8192, 2880], [2880, 2880, 8192])
    assert T.espace_octets(dims, 8) > LIMITE
    desc = T.MoeCouche()
    desc.dims = dims
    desc.k = 8
    desc.experts = 8
    assert T.lib.trc_moe_couche_sans_alloc(C.byref(desc), None) == T.TRC_ERR_USAGE
    assert str(LIMITE) in T.lib.trc_derniere_erreur().decode()


def test_refuse_sans_descripteur():
    assert T.lib.trc_moe_couche_sans_alloc(None, None) == T.TRC_ERR_USAGE
    assert "descriptor" in T.lib.trc_derniere_erreur().decode()


@pytest.mark.gpu
@pytest.mark.parametrize("nom,k", [("couche_petite", 4), ("couche_gpt_oss", 4), ("couche_gpt_oss", 8)])
def test_deux_appels_comme_l_espace_du_demandeur(nom, k, request, noyaux):
    import torch

    from troncons_b200.carte import CoucheCarte

    c = request.getfixturevalue(nom)
    assert T.espace_octets(c.dims, k) <= LIMITE
    cc = CoucheCarte(c, k=k, brut=False)
    rng = np.random.default_rng(31 + k)
    xs, r0s = [], []
    for _ in range(2):
        xf = rng.standard_normal(c.dims.colonnes[0]).astype(np.float32)
        xs.append(torch.from_numpy(xf).to(torch.bfloat16).cuda())
        r0s.append(torch.from_numpy(rng.standard_normal(c.dims.lignes[2]).astype(np.float32)).cuda())

    # The existing entry point, with the workspace the caller allocated.
    attendus = []
    for x, r0 in zip(xs, r0s):
        r = r0.clone()
        cc.controle.zero_()
        cc.couche(x, r)
        torch.cuda.synchronize()
        assert (cc.controle == 0).all()
        attendus.append((r.cpu(), cc.idx.cpu().clone(), cc.poids.cpu().clone()))

    # The fixed workspace: two calls back to back on the same stream.
    obtenus, descs = [], []
    cc.controle.zero_()
    for x, r0 in zip(xs, r0s):
        r = r0.clone()
        cc.routeur(x)
        descs.append(cc.descripteur(x, r, False))
        noyaux.moe_couche_sans_alloc(descs[-1])
        obtenus.append((r, cc.idx.clone(), cc.poids.clone()))
    torch.cuda.synchronize()
    assert (cc.controle == 0).all()
    for i, ((ra, ia, wa), (rb, ib, wb)) in enumerate(zip(attendus, obtenus)):
        assert torch.equal(ia, ib.cpu()) and torch.equal(wa, wb.cpu()), f"call {i}: routing differs"
        assert torch.equal(ra.view(torch.int32), rb.cpu().view(torch.int32)), f"call {i}: residual differs"


@pytest.mark.parametrize("k,jetons,motif", [(9, 1, "k = 9"), (0, 1, "k = 0"), (4, 129, "129 tokens")])
def test_refuse_k_et_jetons_d_abord(k, jetons, motif):
    """A bad k or token count is reported as itself, before the workspace size is worked out."""
    desc = T.MoeCouche()
    desc.dims = T.DimsExpert.de([256, 256, 512], [512, 512, 256])
    desc.k = k
    desc.experts = 8
    desc.jetons = jetons
    assert T.lib.trc_moe_couche_sans_alloc(C.byref(desc), None) == T.TRC_ERR_USAGE
    assert motif in T.lib.trc_derniere_erreur().decode()
