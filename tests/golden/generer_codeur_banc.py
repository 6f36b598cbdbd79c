"""Writes tests/golden/codeur_banc.json: SHA-256 of level-0 parts written by the reference's
own independent encoder (trc-noyaux/banc/banc_k.cu: coder_g1, assembler_partie), compiled
unchanged into oracle/_ref/libtrc_banc.so by `make -C oracle ref`.

Inputs are seeded synthetic experts from troncons_b200.synth.matrices; the frequency tables are
the oracle's normalisation of the layer's counts (the bench's own normalisation is deliberately
different and is not used). Run from the repository root: python tests/golden/generer_codeur_banc.py
"""
import hashlib
import json
import os
import sys

RACINE = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path[:0] = [RACINE, os.path.join(RACINE, "tests")]

import numpy as np  # noqa: E402

import oracle as O  # noqa: E402
import trc_aides as A  # noqa: E402
import troncons_b200 as T  # noqa: E402
import troncons_b200.synth as S  # noqa: E402

CAS = [
    # (seed, lignes, colonnes, experts, canonique, n_delta, n_codes)
    (101, [256, 256, 512], [512, 512, 256], 2, True, 256, 256),
    (102, [256, 256, 512], [512, 512, 256], 2, False, 256, 256),
    (103, [96, 96, 64], [64, 64, 96], 3, True, 32, 64),
    (104, [2880, 2880, 2880], [2880, 2880, 2880], 1, True, 32, 256),
]


def parties_banc(graine, lignes, colonnes, experts, canonique, n_delta, n_codes, codeur, assembleur):
    """Parts of `experts` seeded experts: [(part bytes)], tables u16[3][4][256]."""
    dims = T.DimsExpert.de(lignes, colonnes)
    blocs, biais = [], []
    for j in range(3):
        b, bi = S.matrices(graine * 7 + j, lignes[j], colonnes[j], experts)
        blocs.append(b)
        biais.append(bi)
    preps = [[O.preparer_matrice(blocs[j][x], lignes[j], colonnes[j] // 32, canonique) for x in range(experts)]
             for j in range(3)]
    freqs = np.stack([A.tables_matrice(preps[j]) for j in range(3)])
    parties = []
    for x in range(experts):
        flux = []
        for j in range(3):
            R, nb = lignes[j], lignes[j] * (colonnes[j] // 32)
            flux += A.flux_matrice(preps[j][x], biais[j][x].tobytes(), freqs[j], j, R, nb, n_delta, n_codes, codeur)
        parties.append(assembleur(0, x, flux))
    return dims, blocs, biais, freqs, parties


def main():
    banc = O.banc()
    if banc is None:
        raise SystemExit("oracle/_ref/libtrc_banc.so is absent: run `make -C oracle ref` first")
    sortie = []
    for cas in CAS:
        _, _, _, freqs, parties = parties_banc(*cas, codeur=banc, assembleur=banc.assembler_partie)
        sortie.append({
            "graine": cas[0], "lignes": cas[1], "colonnes": cas[2], "experts": cas[3], "canonique": cas[4],
            "n_delta": cas[5], "n_codes": cas[6],
            "tables_sha256": hashlib.sha256(freqs.astype("<u2").tobytes()).hexdigest(),
            "parties": [{"octets": len(p), "sha256": hashlib.sha256(p).hexdigest()} for p in parties],
        })
    chemin = os.path.join(os.path.dirname(os.path.abspath(__file__)), "codeur_banc.json")
    with open(chemin, "w") as f:
        json.dump({"source": "trc-noyaux/banc/banc_k.cu coder_g1 + assembler_partie (reference, compiled unchanged)",
                   "cas": sortie}, f, indent=1)
    print(chemin)


if __name__ == "__main__":
    main()
