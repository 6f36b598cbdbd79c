"""GPU, one device: the combine's exchange gives up when a rank never arrives, and says so.

The fused layer is called with a two-rank exchange whose "other rank" buffer is a second buffer
on this same GPU (every store stays local): nothing ever raises the other rank's flag, so the
combine's bounded wait runs out (about 1.5 s), the kernel counts it in controle[3] of activation
0, leaves the residual unchanged and returns; the context stays usable (a normal call right
after gives the normal result). No fault, no trap, no endless loop."""
import ctypes as C

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def test_attente_du_rang_absent(couche_petite):
    import troncons_b200 as T
    from troncons_b200.carte import CoucheCarte

    c = couche_petite
    cc = CoucheCarte(c, k=4, brut=False)
    n = T.echange_octets(c.dims, 1, 2)
    tampons = torch.zeros(2, n + 256, dtype=torch.uint8, device="cuda")
    a = [tampons[q].data_ptr() + (-tampons[q].data_ptr()) % 256 for q in range(2)]
    ech = T.EchangePairs((C.c_uint64 * 8)(*(a + [0] * 6)), 0, 2)
    rng = np.random.default_rng(9)
    x = torch.from_numpy(rng.standard_normal(c.dims.colonnes[0]).astype(np.float32)).to(torch.bfloat16).cuda()
    r0 = torch.from_numpy(rng.standard_normal(c.dims.lignes[2]).astype(np.float32)).cuda()
    r = r0.clone()
    cc.controle.zero_()
    cc.couche(x, r, echange=ech)
    torch.cuda.synchronize()
    ctl = cc.controle.cpu().numpy().reshape(-1, 4)
    assert ctl[0, 3] >= 1, "the wait did not report giving up"
    assert torch.equal(r, r0), "the residual changed although the exchange failed"
    # the context is still usable
    r2 = r0.clone()
    cc.controle.zero_()
    cc.couche(x, r2)
    r3 = r0.clone()
    cc.couche(x, r3)
    torch.cuda.synchronize()
    assert (cc.controle == 0).all() or (cc.controle.cpu().numpy().reshape(-1, 4)[:, :3] == 0).all()
    assert torch.equal(r2, r3) and not torch.equal(r2, r0)
