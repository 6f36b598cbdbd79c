"""Writes a JSON fixture of outputs of the reference's own CUDA kernels (trc-noyaux/noyaux/
noyaux.cu compiled unchanged for sm_100a into oracle/_ref/libtrc_ref.so by `make -C oracle ref`),
on seeded synthetic inputs. Needs a GPU; the fixture is committed as tests/golden/noyaux_ref.json
and checked against the CPU oracle by tests/test_golden_noyaux_ref.py, without a GPU.

Recorded:
- decode (decoder_echelles + decoder_codes, abi.rs grids): SHA-256 of the SoA slot of every
  expert of two seeded layers (a small one and one of the gpt-oss-120b shape), with the SHA-256
  of the parts and LUTs they were decoded from, and the integrity counters;
- gemv_mxfp4 on matrices of those slots: y as f32 bits;
- routeur_topk, swiglu_oai, combiner, gemv_f32 on seeded vectors: outputs as f32 / u32 bits.

Usage (repository root, on a GPU box): python tests/golden/generer_noyaux_ref.py <output.json>
"""
import hashlib
import json
import os
import sys

RACINE = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path[:0] = [RACINE]

import numpy as np  # noqa: E402
import torch  # noqa: E402

import oracle as O  # noqa: E402
import troncons_b200 as T  # noqa: E402
import troncons_b200.synth as S  # noqa: E402

COUCHES = [
    # (seed, lignes, colonnes, experts)
    (501, [256, 256, 512], [512, 512, 256], 3),
    (502, [2880, 2880, 2880], [2880, 2880, 2880], 1),
]


def sha(b) -> str:
    return hashlib.sha256(bytes(b)).hexdigest()


def dev(a: np.ndarray) -> torch.Tensor:
    """A device copy. Keep it referenced until the kernel that reads it has completed: a
    temporary whose address was passed on is freed at once, and the caching allocator may hand
    its block to the next copy before the kernel runs."""
    return torch.from_numpy(np.array(a)).cuda()


def bits(t: torch.Tensor) -> list:
    return [int(v) for v in t.cpu().numpy().reshape(-1).view(np.uint32)]


def entrees_gemv_f32(E: int, C: int):
    """The router GEMV's seeded inputs (W f32[E][C], x f32[C], b f32[E])."""
    rng = np.random.default_rng(78)
    W = (rng.standard_normal((E, C)) * 0.02).astype(np.float32)
    xv = rng.standard_normal(C).astype(np.float32)
    b = (rng.standard_normal(E) * 0.01).astype(np.float32)
    return W, xv, b


def main(chemin: str):
    ref = O.ref()
    if ref is None:
        raise SystemExit("oracle/_ref/libtrc_ref.so is absent: run `make -C oracle ref` where the reference is")
    s = torch.cuda.current_stream().cuda_stream
    sortie = {"source": "trc-noyaux/noyaux/noyaux.cu (reference kernels, compiled unchanged for sm_100a)",
              "couches": [], "gemv": [], "topk": [], "swiglu": None, "combiner": None, "gemv_f32": None}
    slots = {}
    for graine, lignes, colonnes, experts in COUCHES:
        c = S.couche(graine, T.DimsExpert.de(lignes, colonnes), experts, brut=False)
        te = T.taille_emplacement(c.dims)
        dims6 = np.array(lignes + colonnes, np.uint32)
        l = dev(c.luts)
        ex = []
        for x in range(experts):
            p = dev(np.frombuffer(c.parties[x], np.uint8))
            e = torch.zeros(te, dtype=torch.uint8, device="cuda")
            ctl = torch.zeros(4, dtype=torch.int32, device="cuda")
            assert ref.ref_decoder_expert(p.data_ptr(), e.data_ptr(), l.data_ptr(), O.p(dims6, O.P32), ctl.data_ptr(),
                                          s) == 0
            torch.cuda.synchronize()
            slots[(graine, x)] = e
            ex.append({"partie_sha256": sha(c.parties[x]), "emplacement_sha256": sha(e.cpu().numpy()),
                       "controle": [int(v) for v in ctl.cpu().numpy()]})
        sortie["couches"].append({"graine": graine, "lignes": lignes, "colonnes": colonnes, "experts": experts,
                                  "luts_sha256": sha(c.luts.astype("<u4").tobytes()), "experts_decodes": ex})

    rng = np.random.default_rng(77)
    for graine, x, j in [(501, 0, 0), (501, 2, 2), (502, 0, 1)]:
        lignes, colonnes = next((cl[1], cl[2]) for cl in COUCHES if cl[0] == graine)
        base = sum(O.disposition(lignes[i], colonnes[i])[2] for i in range(j))
        R, C = lignes[j], colonnes[j]
        xv = rng.standard_normal(C).astype(np.float32)
        y = torch.zeros(R, dtype=torch.float32, device="cuda")
        m = slots[(graine, x)][base:]
        xd = dev(xv)
        assert ref.ref_gemv(m.data_ptr(), xd.data_ptr(), y.data_ptr(), R, C, s) == 0
        torch.cuda.synchronize()
        sortie["gemv"].append({"graine": graine, "expert": x, "matrice": j, "x_bits": bits(torch.from_numpy(xv)),
                               "y_bits": bits(y)})

    for k in (1, 4, 8):
        for cas in range(3):
            lg = rng.standard_normal(128).astype(np.float32)
            if cas == 1:  # ties: repeated values, the smaller index must win
                lg[[5, 17, 90]] = lg.max() + 1.0
            if cas == 2:  # coarse values, many ties
                lg = np.round(lg * 2.0) / 2.0
            idx = torch.zeros(k, dtype=torch.int32, device="cuda")
            w = torch.zeros(k, dtype=torch.float32, device="cuda")
            ld = dev(lg)
            assert ref.ref_routeur_topk(ld.data_ptr(), 128, k, idx.data_ptr(), w.data_ptr(), s) == 0
            torch.cuda.synchronize()
            sortie["topk"].append({"k": k, "logits_bits": bits(torch.from_numpy(lg)),
                                   "indices": [int(v) for v in idx.cpu().numpy()], "poids_bits": bits(w)})

    n = 4096
    g = (rng.standard_normal(n) * 4.0).astype(np.float32)
    u = (rng.standard_normal(n) * 4.0).astype(np.float32)
    g[:8] = [7.0, -7.0, 7.0000005, -7.0000005, 0.0, -0.0, 30.0, -30.0]
    u[:8] = [7.0, -7.0, 6.9999995, -6.9999995, 0.0, -0.0, 30.0, -30.0]
    y = torch.zeros(n, dtype=torch.float32, device="cuda")
    gd, ud = dev(g), dev(u)
    assert ref.ref_swiglu(gd.data_ptr(), ud.data_ptr(), y.data_ptr(), n, s) == 0
    torch.cuda.synchronize()
    sortie["swiglu"] = {"g_bits": bits(torch.from_numpy(g)), "u_bits": bits(torch.from_numpy(u)), "y_bits": bits(y)}

    d, kk = 2880, 4
    res = rng.standard_normal(d).astype(np.float32)
    so = rng.standard_normal((kk, d)).astype(np.float32)
    w = rng.random(kk).astype(np.float32)
    r = dev(res)
    sd, wd = dev(so), dev(w)
    assert ref.ref_combiner(r.data_ptr(), sd.data_ptr(), d, wd.data_ptr(), kk, d, s) == 0
    torch.cuda.synchronize()
    sortie["combiner"] = {"residu_bits": bits(torch.from_numpy(res)), "sorties_bits": bits(torch.from_numpy(so)),
                          "poids_bits": bits(torch.from_numpy(w)), "sortie_bits": bits(r)}

    E, C = 128, 2880
    W, xv, b = entrees_gemv_f32(E, C)
    y = torch.zeros(E, dtype=torch.float32, device="cuda")
    Wd, xd, bd = dev(W), dev(xv), dev(b)
    assert ref.ref_gemv_f32(Wd.data_ptr(), xd.data_ptr(), bd.data_ptr(), y.data_ptr(), E, C, s) == 0
    torch.cuda.synchronize()
    sortie["gemv_f32"] = {"graine_numpy": 78, "W_sha256": sha(W.tobytes()), "x_bits": bits(torch.from_numpy(xv)),
                          "b_bits": bits(torch.from_numpy(b)), "y_bits": bits(y)}

    with open(chemin, "w") as f:
        json.dump(sortie, f)
    print(chemin)


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.path.join(os.path.dirname(os.path.abspath(__file__)),
                                                              "noyaux_ref.json"))
