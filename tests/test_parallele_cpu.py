"""CPU: the expert-parallel host logic (troncons_b200/parallele.py), with two `gloo` ranks.

- shares are contiguous, disjoint, cover every expert, and differ in size by at most one;
- two ranks that each draw and encode only their experts, summing the layer's counts with an
  all-reduce, build exactly the single-process layer: same tables, same parts, byte for byte;
- one expert-parallel step (rank 0 adds its share into the residual, the other writes its share
  alone, then a SUM all-reduce) gives both ranks the whole layer's result, on a small dense MoE
  computed in numpy (the same terms as a single process, summed in another order: 1e-6)."""
import os
import socket
from datetime import timedelta

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from troncons_b200.parallele import partage  # noqa: E402


@pytest.mark.parametrize("experts", [128, 8, 10, 129])
@pytest.mark.parametrize("monde", [1, 2, 3, 4, 8])
def test_partage(experts, monde):
    s = [partage(experts, r, monde) for r in range(monde)]
    assert s[0][0] == 0 and s[-1][1] == experts
    assert all(a[1] == b[0] for a, b in zip(s, s[1:]))
    tailles = [f - d for d, f in s]
    assert max(tailles) - min(tailles) <= 1 and min(tailles) >= 1


def test_partage_refuse():
    with pytest.raises(ValueError):
        partage(4, 0, 8)
    with pytest.raises(ValueError):
        partage(8, 2, 2)


def _port_libre() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _moe_dense(rng, E, d, jetons, k):
    W = rng.standard_normal((E, d, d)).astype(np.float32)
    Wr = rng.standard_normal((E, d)).astype(np.float32)
    x = rng.standard_normal((jetons, d)).astype(np.float32)
    r0 = rng.standard_normal((jetons, d)).astype(np.float32)
    logits = x @ Wr.T
    idx = np.argsort(-logits, axis=1, kind="stable")[:, :k]
    w = np.exp(np.take_along_axis(logits, idx, 1) - logits.max(1, keepdims=True))
    w = (w / w.sum(1, keepdims=True)).astype(np.float32)
    return W, x, r0, idx, w


def _somme_locale(W, x, idx, w, debut, fin):
    """Per token, the slot-ordered weighted sum over the activations whose expert is held."""
    jetons, d = x.shape
    s = np.zeros((jetons, d), np.float32)
    for b in range(jetons):
        premier = True
        for u in range(idx.shape[1]):
            e = int(idx[b, u])
            if not debut <= e < fin:
                continue
            p = np.float32(w[b, u]) * (W[e] @ x[b]).astype(np.float32)
            s[b] = p if premier else s[b] + p
            premier = False
    return s


def _travail(rang, monde, port):
    import torch.distributed as dist

    import troncons_b200 as T
    import troncons_b200.synth as S
    from troncons_b200.parallele import etape_ep, reduire_comptes

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rang, world_size=monde,
                            timeout=timedelta(seconds=60))
    try:
        # 1. the layer drawn by shares equals the layer drawn at once
        dims = T.DimsExpert.de([64, 64, 96], [96, 96, 64])
        tenus = partage(8, rang, monde)
        part = S.couche(41, dims, 8, brut=False, tenus=tenus, reduire=reduire_comptes(), fils=2)
        toute = S.couche(41, dims, 8, brut=False, fils=2)
        assert (part.freqs == toute.freqs).all(), "tables differ"
        for e in range(8):
            if tenus[0] <= e < tenus[1]:
                assert part.parties[e] == toute.parties[e], f"part of expert {e} differs"
            else:
                assert part.parties[e] is None

        # 2. one expert-parallel step on a small dense MoE
        rng = np.random.default_rng(7)  # the same draw on every rank
        W, x, r0, idx, w = _moe_dense(rng, 8, 16, 3, 4)
        residu = torch.from_numpy(r0.copy())

        def local(r, partiel):
            s = torch.from_numpy(_somme_locale(W, x, idx, w, *tenus))
            if partiel:
                r.copy_(s)
            else:
                r.add_(s)

        etape_ep(local, residu, rang)
        attendu = r0 + _somme_locale(W, x, idx, w, 0, 8)
        assert np.abs(residu.numpy() - attendu).max() <= 1e-6 * max(1.0, np.abs(attendu).max()) * 8
    finally:
        dist.destroy_process_group()


def test_deux_rangs_gloo():
    import torch.multiprocessing as mp

    port = _port_libre()
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    mp.start_processes(_travail, args=(2, port), nprocs=2, join=True, start_method="spawn")


@pytest.mark.parametrize("placement", ["aleatoire", "equilibre"])
def test_popularite_zipf(placement):
    """The router bias of a Zipf(s)-skewed synthetic model: -s ln(1 + q) for popularity rank q,
    every rank used once; "equilibre" puts the monde most popular experts on monde different
    shares, share r holding exactly the ranks q = r mod monde; "aleatoire" a seeded
    permutation, different per layer."""
    from troncons_b200.modele import biais_zipf

    E, monde, s = 128, 8, 1.1
    b = biais_zipf(E, s, placement, monde, 7, 3)
    assert b.dtype == np.float32 and b.shape == (E,)
    assert np.allclose(np.sort(b)[::-1], -s * np.log1p(np.arange(E)), rtol=0, atol=1e-6)
    ordre = np.argsort(-b, kind="stable")
    parts = [partage(E, r, monde) for r in range(monde)]
    rang_de = lambda e: next(r for r, (d, f) in enumerate(parts) if d <= e < f)  # noqa: E731
    if placement == "equilibre":
        assert sorted(rang_de(int(e)) for e in ordre[:monde]) == list(range(monde))
        for r, (d, f) in enumerate(parts):
            q = sorted(int(np.where(ordre == e)[0][0]) for e in range(d, f))
            assert all(x % monde == r for x in q)
    else:
        assert not np.array_equal(b, biais_zipf(E, s, placement, monde, 7, 4))
    with pytest.raises(ValueError):
        biais_zipf(E, s, "autre", monde, 7, 3)


@pytest.mark.parametrize("kw,motif", [
    (dict(echange="autre"), "exchange"),
    (dict(par_rang=0), "sequences per rank"),
    (dict(par_rang=65, monde=2), "128 tokens"),
    (dict(moe="autre"), "MoE form"),
    (dict(moe="par_flux", echange="pairs", monde=2), "MoE form"),
])
def test_modele_ep_refuse(kw, motif):
    """The expert-parallel model's arguments are checked before anything is drawn on a device:
    the exchange, the sequences per rank (1 to 128 tokens per step over the ranks), the MoE form
    (par flux has no peer-store exchange)."""
    from troncons_b200.parallele import ModeleEP

    monde = kw.pop("monde", 1)
    with pytest.raises(ValueError, match=motif):
        ModeleEP(0, monde, experts=8, **kw)


class _CarteFactice:
    """Stands in for CoucheCarte (which uploads to a GPU): records what the layer asks of it."""

    def __init__(self, c, k, brut, jetons, tenus):
        self.k, self.jetons, self.tenus, self.appels = k, jetons, tenus, []

    def couche(self, x, residu, flux=None, partiel=False, echange=None):
        self.appels.append(("fusionnee", partiel, echange))

    def couche_par_flux(self, x, residu, flux=None, partiel=False):
        self.appels.append(("par_flux", partiel, None))


def _couche_factice(experts=128):
    from types import SimpleNamespace

    return SimpleNamespace(experts=experts, dims=None)


@pytest.mark.parametrize("kw,motif", [
    (dict(echange="autre"), "exchange"),
    (dict(moe="autre"), "MoE form"),
    (dict(moe="par_flux", echange="pairs", monde=2), "MoE form"),
    (dict(k=9), "k = 9"),
    (dict(k=0), "k = 0"),
    (dict(jetons=0), "tokens"),
    (dict(rang=2, monde=2), "rank 2 of 2"),
])
def test_couche_ep_refuse(kw, motif, monkeypatch):
    """The expert-parallel layer refuses bad arguments before any device work (its CoucheCarte
    is never built)."""
    import troncons_b200.carte as carte
    from troncons_b200.parallele import CoucheEP

    monkeypatch.setattr(carte, "CoucheCarte", lambda *a, **k: pytest.fail("device work before the checks"))
    rang, monde = kw.pop("rang", 0), kw.pop("monde", 1)
    with pytest.raises(ValueError, match=motif):
        CoucheEP(_couche_factice(), rang, monde, **kw)


@pytest.mark.parametrize("argv,forme,echange", [
    (["--gpus", "2"], "fusionnee", "pairs"),
    (["--gpus", "2", "--echange", "nccl", "--moe", "par_flux"], "par_flux", "nccl"),
    (["--gpus", "8", "--echange", "nccl"], "fusionnee", "nccl"),
])
def test_bras_ep_construit_la_couche(argv, forme, echange, monkeypatch):
    """bench.py's expert-parallel arm builds its layer from the command line (the path every
    `bench.py --gpus N` run with N > 1 takes) and steps it: the share, the exchange and the MoE
    form reach the layer, the right half of the layer runs. CoucheCarte and the symmetric-memory
    rendezvous are replaced by fakes, so no GPU is needed."""
    import bench
    import troncons_b200.carte as carte
    import troncons_b200.parallele as P

    monkeypatch.setattr(carte, "CoucheCarte", _CarteFactice)
    monkeypatch.setattr(P, "monter_paires", lambda dims, jetons, r, w, g=None: (None, None, "paires"))
    args = bench.arguments(argv)
    w = args.gpus
    for r in (0, w - 1):
        ep = bench.couche_ep(args, _couche_factice(args.experts), r, w)
        assert ep.carte.tenus == P.partage(128, r, w) and ep.carte.jetons == w and ep.carte.k == args.k
        assert ep.echange == echange and ep.moe == forme
        if echange == "pairs":
            ep.etape(None, None)
            assert ep.carte.appels == [("fusionnee", False, "paires")]
        else:
            ep.local(None, None, r != 0)
            assert ep.carte.appels == [(forme, r != 0, None)]
