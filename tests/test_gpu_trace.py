"""GPU: the routing trace (QE_TRACE) of qe_moe_forward in the reference's record format.

The reference's moe_layer_step appends, per token, int32 layer followed by the top-k expert ids as int32 to the
file named by QE_TRACE (engine/src/moe_layer.c:57-64, opened once per process). The Mode R goldens hold the
routing the reference's own trace recorded for synthetic checkpoints; here the library writes its trace for the
same checkpoint and inputs, and the two files must be identical byte for byte (the layer id set at create time
included). QE_TRACE is read once per process, so each case runs in a child process.
"""
import json
import os
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

import oracle as O
from golden_io import checkpoint_tensors, moe_goldens, read_moe_golden, write_safetensors

pytestmark = pytest.mark.gpu

REPO = Path(__file__).resolve().parents[1]
PREFIX = "language_model.model.layers.0.mlp"

CHILD = r"""
import json, sys
import numpy as np
sys.path.insert(0, sys.argv[1])
import qmoe
a = json.loads(sys.argv[2])
x = np.load(a["x"])
blk = qmoe.MoeBlock.from_safetensors(a["dir"], a["prefix"], top_k=a["top_k"], group_size=a["gs"], layer=a["layer"])
for t0 in range(0, x.shape[0], a["chunk"]):        # several calls: the records append in call order
    blk.forward(np.ascontiguousarray(x[t0:t0 + a["chunk"]]))
blk.close()
"""


@pytest.mark.parametrize("layer,chunk", [(0, 1), (7, 2)])
@pytest.mark.parametrize("path", [p for p in moe_goldens() if read_moe_golden(p)["mode"] == "R"], ids=lambda p: p.stem)
def test_trace_matches_reference_records(path, layer, chunk, tmp_path):
    g = read_moe_golden(path)
    oc = O.SynthBlock(O.BlockCfg(**g["cfg"]), g["seed"], 0, g["bias"])
    write_safetensors(tmp_path / "model.safetensors", checkpoint_tensors(PREFIX, oc.arrays()))
    x = oc.x(g["T"])
    np.save(tmp_path / "x.npy", x)
    trace = tmp_path / "trace.bin"
    args = {"x": str(tmp_path / "x.npy"), "dir": str(tmp_path), "prefix": PREFIX, "top_k": g["cfg"]["top_k"],
            "gs": g["cfg"].get("group_size", 64), "layer": layer, "chunk": chunk}
    env = dict(os.environ, QE_TRACE=str(trace))
    r = subprocess.run([sys.executable, "-c", CHILD, str(REPO / "moe-stream-mac_b200"), json.dumps(args)], env=env,
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    k = g["cfg"]["top_k"]
    want = np.empty((g["T"], 1 + k), np.int32)   # the reference's record: int32 layer, int32 idx[k]
    want[:, 0] = layer
    want[:, 1:] = g["idx"]
    assert trace.read_bytes() == want.tobytes()
