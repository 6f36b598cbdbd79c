"""Writes tests/golden/traces_boucle.npz + traces_boucle.json: two routing traces the reference's
engine wrote (gpt-oss-120b and gpt-oss-20b, 708 tokens each: mesures/moteur/epreuve-J1/journaux/
programme/invite/t120-boucle.trace, t20-boucle.trace) and the cache counts the reference measured
on them: its engine's own counters (the run's journal, t*-boucle.json "compteurs") and its
simulator's replay (mesures/moteur/O/corrections/journaux/m5-rejouer-invite-326-314.jsonl).
Run here, where the reference is mounted:  python tests/golden/generer_traces.py"""
import json
import os
import sys

import numpy as np

ICI = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ICI, "..", ".."))
REF = os.path.join(os.environ.get("TRONCONS_REF", "/root/reference"), "mesures", "moteur")


def main():
    from troncons_b200.cache import lire_trace

    tableaux, attendus = {}, {}
    for nom in ("t120-boucle", "t20-boucle"):
        base = os.path.join(REF, "epreuve-J1/journaux/programme/invite", nom)
        tr = lire_trace(base + ".trace")
        assert tr.experts <= 256
        tableaux[nom] = tr.choix.astype(np.uint8)
        with open(base + ".json") as f:
            cpt = json.load(f)["compteurs"]
        attendus[nom] = {"experts": tr.experts, "resultats": [
            {k: cpt[k] for k in ("emplacements", "tiedes", "acces", "succes_vram", "succes_ram", "defauts_disque",
                                 "evictions")} | {"source": f"{nom}.json (engine counters)"}]}
    with open(os.path.join(REF, "O/corrections/journaux/m5-rejouer-invite-326-314.jsonl")) as f:
        for ligne in f:
            d = json.loads(ligne)
            nom = os.path.basename(d["trace"]).replace(".trace", "")
            for r in d["resultats"]:
                attendus[nom]["resultats"].append(dict(r) | {"politique": d["politique"], "casser": d["casser"],
                                                             "source": "m5-rejouer-invite-326-314.jsonl (rejouer)"})
    np.savez_compressed(os.path.join(ICI, "traces_boucle.npz"), **{k.replace("-", "_"): v for k, v in tableaux.items()})
    with open(os.path.join(ICI, "traces_boucle.json"), "w") as f:
        json.dump(attendus, f, indent=1)
    print({k: v.shape for k, v in tableaux.items()})


if __name__ == "__main__":
    main()
