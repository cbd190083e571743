"""Loading of the golden fixtures (written by tests/golden/make_golden.py from the
reference code) and regeneration of their seeded inputs."""
import glob
import os

import numpy as np
import torch

from oracle import bsa_oracle as O

GOLDEN_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def fixture_names():
    return sorted(os.path.basename(p)[:-4] for p in glob.glob(os.path.join(GOLDEN_DIR, "*.npz")))


def load(name):
    z = np.load(os.path.join(GOLDEN_DIR, name + ".npz"))
    d = {k: z[k] for k in z.files}
    B, N, Hq, Hk, bs, K, bas, seed = (int(x) for x in d["meta"])
    d.update(B=B, N=N, Hq=Hq, Hk=Hk, bs=bs, K=K, bas=bas, seed=seed)
    return d


def inputs(d):
    """The fixture's inputs, drawn exactly as make_golden.py drew them."""
    return O.make_inputs(d["B"], d["N"], d["Hq"], d["Hk"], seed=d["seed"], rope=True)


def t(a):
    return torch.from_numpy(np.asarray(a)).float()
