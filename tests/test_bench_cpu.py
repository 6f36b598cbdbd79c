"""CPU: bench.py's reference arm and its CPU legs.

- `bench.py --impl reference` prints its JSON line (the config-1 keys of the GPU arm, a
  cpu_baseline, e2e with zero copies, config 0's decode figure) without loading the product
  library: its layer comes from the oracle alone;
- the two arms draw the same inputs (x rounded to bf16, the same residuals);
- config 0's CPU decode covers one gate + up pair: 8,812,800 decoded bytes at 2880 x 2880."""
import json
import os
import subprocess
import sys

import numpy as np

RACINE = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

SONDE = r"""
import json, sys
sys.argv = ["bench.py", "--impl", "reference", "--experts", "6", "--steps", "2", "--warmup", "1"]
import bench
bench.main()
cartes = open("/proc/self/maps").read()
print(json.dumps({"produit_charge": "libtroncons_b200" in cartes or "troncons_b200" in sys.modules}))
"""


def test_bras_reference_sans_le_produit():
    r = subprocess.run([sys.executable, "-c", SONDE], cwd=RACINE, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    lignes = [json.loads(l) for l in r.stdout.splitlines() if l.startswith("{")]
    ligne, sonde = lignes[0], lignes[-1]
    assert sonde == {"produit_charge": False}
    assert ligne["impl"] == "reference" and ligne["value"] > 0 and ligne["steps"] == 2
    assert ligne["e2e"]["h2d_bytes_per_step"] == 0 and ligne["e2e"]["value"] == ligne["value"]
    assert ligne["cpu_baseline"]["kind"] == "port" and ligne["cpu_baseline"]["cores"] >= 1
    import bench

    attendu = bench.config_couche(bench.arguments(["--experts", "6"]), "", "")
    assert set(attendu) <= set(ligne["config"]) and ligne["config"]["workload"] == attendu["workload"]
    c0 = ligne["config0"]
    assert c0["decoded_bytes_per_pair"] == 8812800 and c0["value"] > 0 and c0["nproc"] >= 1


def test_memes_entrees_bf16():
    import bench

    args = bench.arguments(["--steps", "3", "--warmup", "2"])
    xs, res = bench.entrees_couche(args, 2880, 2880)
    xs2, res2 = bench.entrees_couche(args, 2880, 2880)
    assert xs.shape == (5, 2880) and res.shape == (5, 2880)
    assert np.array_equal(xs, xs2) and np.array_equal(res, res2)
    assert (xs.view(np.uint32) & 0xFFFF == 0).all()  # bf16 values
