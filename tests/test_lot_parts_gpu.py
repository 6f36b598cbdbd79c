"""GPU: the fused layer on a batch of tokens, and split into expert shares (expert parallelism).

- a batch of 3 tokens gives each token, bit for bit, what the single-token layer gives it
  (activations are independent; each token's combine keeps the slot order);
- two shares of the experts, [0, E/2) adding into the residual and [E/2, E) partial (writing
  only its own weighted sum): residual_A + sum_B equals the whole layer within
  1e-5 max|residual| (the same f32 terms summed in another order, as an all-reduce does);
  the parts of the experts a share does not hold are absent (never read);
- a share that holds none of a token's experts leaves its residual unchanged, or writes 0 for
  it when partial."""
import dataclasses

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def _x_r(rng, c, n):
    x = torch.from_numpy(rng.standard_normal((n, c.dims.colonnes[0])).astype(np.float32)).to(torch.bfloat16).cuda()
    r = torch.from_numpy(rng.standard_normal((n, c.dims.lignes[2])).astype(np.float32)).cuda()
    return x.contiguous(), r.contiguous()


@pytest.mark.parametrize("nom", ["couche_petite", "couche_gpt_oss"])
def test_lot_egale_jeton_par_jeton(nom, request):
    from troncons_b200.carte import CoucheCarte

    c = request.getfixturevalue(nom)
    c3 = CoucheCarte(c, k=4, brut=False, jetons=3)
    c1 = CoucheCarte(c, k=4, brut=False)
    rng = np.random.default_rng(12)
    for _ in range(3):
        x, r0 = _x_r(rng, c, 3)
        r3 = r0.clone()
        c3.controle.zero_()
        c3.couche(x, r3)
        torch.cuda.synchronize()
        assert (c3.controle == 0).all()
        for b in range(3):
            r1 = r0[b].clone()
            c1.controle.zero_()
            c1.couche(x[b].contiguous(), r1)
            torch.cuda.synchronize()
            assert (c1.controle == 0).all()
            assert torch.equal(c3.idx[4 * b:4 * b + 4], c1.idx)
            assert torch.equal(r3[b].view(torch.int32), r1.view(torch.int32)), f"token {b}"


def _part(c, debut, fin):
    """The same layer with only experts [debut, fin) present."""
    return dataclasses.replace(c, parties=[p if debut <= e < fin else None for e, p in enumerate(c.parties)],
                               parties_brutes=[])


def test_deux_parts_somment_la_couche(couche_petite):
    from troncons_b200.carte import CoucheCarte

    c = couche_petite
    E = c.experts
    toute = CoucheCarte(c, k=4, brut=False, jetons=2)
    a = CoucheCarte(_part(c, 0, E // 2), k=4, brut=False, jetons=2, tenus=(0, E // 2))
    b = CoucheCarte(_part(c, E // 2, E), k=4, brut=False, jetons=2, tenus=(E // 2, E))
    rng = np.random.default_rng(21)
    for _ in range(8):
        x, r0 = _x_r(rng, c, 2)
        rt, ra = r0.clone(), r0.clone()
        rb = torch.full_like(r0, 123.0)
        for cc in (toute, a, b):
            cc.controle.zero_()
        toute.couche(x, rt)
        a.couche(x, ra)
        b.couche(x, rb, partiel=True)
        torch.cuda.synchronize()
        for cc in (toute, a, b):
            assert (cc.controle == 0).all()
        assert torch.equal(a.idx, toute.idx) and torch.equal(b.idx, toute.idx)
        somme = (ra + rb).cpu().numpy()
        attendu = rt.cpu().numpy()
        assert np.abs(somme - attendu).max() <= 1e-5 * max(1.0, np.abs(attendu).max())


def test_part_sans_expert_du_jeton(couche_petite):
    from troncons_b200.carte import CoucheCarte

    c = couche_petite
    toute = CoucheCarte(c, k=4, brut=False)
    rng = np.random.default_rng(5)
    x, r0 = _x_r(rng, c, 1)
    toute.routeur(x)
    torch.cuda.synchronize()
    absents = sorted(set(range(c.experts)) - set(int(v) for v in toute.idx.cpu().numpy()))
    e = absents[0]
    p = CoucheCarte(_part(c, e, e + 1), k=4, brut=False, tenus=(e, e + 1))
    r = r0.clone()
    p.couche(x, r)
    q = torch.full_like(r0, 7.0)
    p.couche(x, q, partiel=True)
    torch.cuda.synchronize()
    assert torch.equal(r, r0)
    assert (q == 0).all()
