"""The backbone's decode attention at the real head layout (32 query and 8 kv heads of 64, four
query heads per kv head) on the tensor cores, against the scalar f32 kernel that implements the
same contract (needs a B200).

The tiny model's backbone has two query heads per kv head; this test runs the depth-sized
synthetic model, whose one backbone layer has the full model's attention shape, so the 16-row
query tile holds four heads and sessions of a few hundred cached positions cover several
64-position chunks and the split-range combine (8 ranges per session at this batch size, some
of them empty). Each kernel runs in its own process (the choice is made once per process); one
decode step after identical batched creations must leave the same final hidden states within
the parity tolerance: the tensor-core kernel rounds the queries and the probabilities to f16,
the scalar kernel keeps them in f32.
"""
import os
import subprocess
import sys

import numpy as np
import pytest

from parity_helpers import LOGIT_ATOL

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
COS_MIN = 0.9995

_SCRIPT = r"""
import sys
import numpy as np
sys.path.insert(0, sys.argv[1])
import __graft_entry__ as g
pkg = g.load_package()
gen = pkg.GeneratorHandle(sys.argv[2], 0)
rng = np.random.default_rng(11)
specs = []
for i, n in enumerate([3, 40, 150, 260, 410, 520]):
    ids = rng.integers(300, 20000, n).tolist()
    specs.append(dict(session_id=50 + i, text=pkg.ids_to_text(ids), seed=i, max_new_tokens=8))
gen.sessions_create_batch(specs)
ids = [sp["session_id"] for sp in specs]
gen.sessions_step_batched(ids, seeds=[7 + i for i in range(len(ids))])
h = np.stack([gen.debug_hidden(sid, 2048) for sid in ids])  # the full model's backbone width
np.save(sys.argv[3], h)
gen.close()
"""


@pytest.fixture(scope="module")
def depth_model(pkg, model_dir):
    return pkg.synth_model(str(model_dir / "depth_nc8.gguf"), preset="depth", nc=8, seed=5)


def _run(depth_model, tmp_path, mma):
    out = str(tmp_path / f"hidden_{mma}.npy")
    env = dict(os.environ, BZB_ATTN_MMA=str(mma))
    r = subprocess.run([sys.executable, "-c", _SCRIPT, ROOT, depth_model, out], env=env, capture_output=True,
                       text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    return np.load(out)


def test_tensor_core_decode_attention_matches_scalar_kernel(depth_model, tmp_path):
    h_mma = _run(depth_model, tmp_path, 1)
    h_ref = _run(depth_model, tmp_path, 0)
    assert h_mma.shape == h_ref.shape and np.isfinite(h_mma).all()
    for i in range(h_ref.shape[0]):
        a, b = h_mma[i].astype(np.float64), h_ref[i].astype(np.float64)
        cos = float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b) + 1e-30))
        assert np.abs(a - b).max() < LOGIT_ATOL and cos > COS_MIN, (i, np.abs(a - b).max(), cos)
