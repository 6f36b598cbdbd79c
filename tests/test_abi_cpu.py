"""CPU: the C-ABI boundary without a GPU.

- the library loads and exports every function include/troncons_b200.h declares;
- the header's structs have the reference's frozen sizes (DimsExpert 24 B, DescGemv 32 B,
  DescDecodage 32 B, ParamsRope 48 B, ParamsAttention 32 B: trc-noyaux/src/abi.rs:305-323) and the Python mirrors have the header's
  layout, field by field (a C program compiled against the header prints sizeof / offsetof);
- bad sizes, shapes and alignments are refused with TRC_ERR_USAGE and a message, before
  anything is launched, as `Noyaux` refuses them with `Erreur::Usage`
  (trc-noyaux/src/lib.rs:70-72, 127-135, 240-245)."""
import ctypes as C
import os
import re
import shutil
import subprocess

import pytest

import troncons_b200 as T
import troncons_b200.juge as J

RACINE = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
ENTETE = os.path.join(RACINE, "include", "troncons_b200.h")


def _fonctions_declarees():
    texte = open(ENTETE).read()
    texte = re.sub(r"/\*.*?\*/", "", texte, flags=re.S)
    return sorted(set(re.findall(r"\b(trc_\w+)\s*\(", texte)))


def test_la_bibliotheque_exporte_tout_l_entete():
    noms = _fonctions_declarees()
    assert len(noms) >= 23
    absents = [n for n in noms if not hasattr(T.lib, n)]
    assert not absents, f"declared but not exported: {absents}"
    if shutil.which("nm"):
        so = T.lib._name
        sortie = subprocess.run(["nm", "-D", "--defined-only", so], check=True, capture_output=True, text=True).stdout
        exportes = sorted({l.split()[-1] for l in sortie.splitlines() if l.split()[-1].startswith("trc_")})
        assert exportes == noms, "exported trc_ symbols differ from the header's declarations"


_STRUCTS = {
    "trc_dims_expert": (T.DimsExpert, 24),
    "trc_desc_gemv": (T.DescGemv, 32),
    "trc_desc_decodage": (T.DescDecodage, 32),
    "trc_moe_couche": (T.MoeCouche, None),
    "trc_params_rope": (T.ParamsRope, 48),
    "trc_params_attention": (T.ParamsAttention, 32),
    "trc_juge_position": (J.JugePosition, 48),
    "trc_desc_gemm": (T.DescGemm, 56),
}


@pytest.mark.skipif(shutil.which("gcc") is None, reason="no C compiler")
def test_disposition_des_structures(tmp_path):
    lignes = ['#include <stdio.h>', '#include <stddef.h>', '#include "troncons_b200.h"', "int main(void) {"]
    for nom, (py, _) in _STRUCTS.items():
        lignes.append(f'printf("{nom} sizeof %zu\\n", sizeof({nom}));')
        for champ, _ in py._fields_:
            lignes.append(f'printf("{nom} {champ} %zu\\n", offsetof({nom}, {champ}));')
    lignes.append("return 0; }")
    src = tmp_path / "disposition.c"
    src.write_text("\n".join(lignes))
    exe = tmp_path / "disposition"
    subprocess.run(["gcc", "-std=c11", "-I", os.path.dirname(ENTETE), "-o", str(exe), str(src)], check=True)
    sortie = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.split("\n")
    vu = {}
    for l in sortie:
        if l:
            s, c, v = l.split()
            vu[(s, c)] = int(v)
    for nom, (py, taille) in _STRUCTS.items():
        assert vu[(nom, "sizeof")] == C.sizeof(py), nom
        if taille is not None:
            assert C.sizeof(py) == taille, nom
        for champ, _ in py._fields_:
            assert vu[(nom, champ)] == getattr(py, champ).offset, f"{nom}.{champ}"


def _erreur():
    return T.lib.trc_derniere_erreur().decode()


def test_refus_gemv():
    # Columns not a multiple of 32.
    assert T.lib.trc_gemv(None, 0, None, 0, None, 0, 64, 33, None) == T.TRC_ERR_USAGE
    assert "33" in _erreur()


def test_refus_decodage():
    d = T.DimsExpert.gpt_oss()
    # A part smaller than its header.
    assert T.lib.trc_decoder_expert(None, 0, C.c_void_p(256), 13_254_144, None, 0, C.byref(d), None, 0,
                                    None) == T.TRC_ERR_USAGE
    # A misaligned slot, with an otherwise plausible part.
    assert T.lib.trc_decoder_expert(C.c_void_p(4096), 8192, C.c_void_p(257), 13_254_144, C.c_void_p(4096),
                                    196_608, C.byref(d), C.c_void_p(4096), 16, None) == T.TRC_ERR_USAGE
    # A slot that is too small.
    assert T.lib.trc_decoder_expert(C.c_void_p(4096), 8192, C.c_void_p(256), 13_254_143, C.c_void_p(4096),
                                    196_608, C.byref(d), C.c_void_p(4096), 16, None) == T.TRC_ERR_USAGE


def test_refus_routeur_topk():
    # k above 8.
    assert T.lib.trc_routeur_topk(C.c_void_p(256), 512, 128, 9, C.c_void_p(256), 64, C.c_void_p(256), 64, 0, 0,
                                  None) == T.TRC_ERR_USAGE


def _couche(**kw):
    d = T.MoeCouche()
    d.parties = d.parties_octets = d.indices = d.poids = d.x = d.residu = d.controle = d.luts = 4096
    d.experts, d.k = 128, 4
    d.dims = T.DimsExpert.gpt_oss()
    for k, v in kw.items():
        setattr(d, k, v)
    return d


@pytest.mark.parametrize("champs,mot", [
    ({"k": 0}, "k = 0"),
    ({"k": 9}, "k = 9"),
    ({"dims": T.DimsExpert.de([2880, 2880, 2880], [2880, 2880, 1440])}, "chain"),
    ({"x": 4098}, "misaligned"),
    ({"residu": None}, "missing"),
])
def test_refus_couche(champs, mot):
    d = _couche(**champs)
    e = T.espace_octets(T.DimsExpert.gpt_oss(), 4)
    assert T.lib.trc_moe_couche_fusionnee(C.byref(d), C.c_void_p(1 << 20), e, None) == T.TRC_ERR_USAGE
    assert mot in _erreur()


def test_refus_espace_trop_petit():
    d = _couche()
    e = T.espace_octets(T.DimsExpert.gpt_oss(), 4)
    assert T.lib.trc_moe_couche_fusionnee(C.byref(d), C.c_void_p(1 << 20), e - 1, None) == T.TRC_ERR_USAGE
    assert "workspace" in _erreur()
    assert T.lib.trc_moe_couche_fusionnee(C.byref(d), C.c_void_p((1 << 20) + 16), e, None) == T.TRC_ERR_USAGE


def test_espace_grandit_avec_k():
    d = T.DimsExpert.gpt_oss()
    e = [T.espace_octets(d, k) for k in range(1, 9)]
    assert all(b > a for a, b in zip(e, e[1:]))
    assert e[3] == 3_432_960 and e[7] == 6_865_920


def test_refus_attention():
    import troncons_b200 as T2

    p = T2.ParamsAttention.gpt_oss(300, 128)
    p.dim_tete = 32
    v = C.c_void_p(4096)
    assert T.lib.trc_attention(v, 1 << 20, v, 1 << 20, v, 1 << 20, v, 1 << 20, v, 1 << 20, C.byref(p), None) == T.TRC_ERR_USAGE
    p = T2.ParamsAttention.gpt_oss(300, 128)
    p.debut = 0  # 301 positions in a ring of 128 cases
    assert T.lib.trc_attention(v, 1 << 20, v, 1 << 20, v, 1 << 20, v, 1 << 20, v, 1 << 20, C.byref(p), None) == T.TRC_ERR_USAGE
    assert "ring" in _erreur()
    r = T2.ParamsRope.gpt_oss()
    r.dim_tete = 65
    assert T.lib.trc_rope_yarn(v, 1 << 20, v, 1 << 20, 64, 8, 0, C.byref(r), None) == T.TRC_ERR_USAGE
    # a KV case past the cache
    assert T.lib.trc_ecrire_kv(v, 2048, v, 2048, v, 1024, v, 1024, 512, 1, None) == T.TRC_ERR_USAGE


def test_refus_couche_ep():
    """The expert-parallel entry refuses, before touching a device or NCCL, a missing
    communicator and a descriptor that sets the partial combine or the peer exchange itself."""
    import ctypes as C

    desc = T.MoeCouche()
    assert T.lib.trc_moe_couche_ep(C.byref(desc), None, 0, None, None) == T.TRC_ERR_USAGE
    desc.partiel = 1
    assert T.lib.trc_moe_couche_ep(C.byref(desc), None, 0, C.c_void_p(1), None) == T.TRC_ERR_USAGE
    assert "partiel" in T.lib.trc_derniere_erreur().decode()
    ident = (C.c_uint8 * 128)()
    assert T.lib.trc_nccl_id(ident, 64) == T.TRC_ERR_USAGE
    assert T.lib.trc_nccl_init(None, 2, ident, 2) == T.TRC_ERR_USAGE
