"""Row-sharded dense layer over 2 GPUs with a single-device result requested:
dense_rows(gather=True) assembles Y on every rank slab by slab while later
slabs compute, by peer DMA into IPC-mapped buffers (transport "ce"), by
NCCL all-gather (transport "nccl"), by the GEMM epilogue's own stores into
the peers' buffers (transport "fused"), or by its stores to an NVSwitch
multicast address (transport "multimem"). Run as 2 ranks under torchrun; skipped with fewer
than 2 GPUs."""
import os
import socket
import subprocess
import sys

import pytest

from conftest import PKG_PARENT, ROOT

pytestmark = pytest.mark.gpu

_SCRIPT = r"""
import os, sys, ctypes
sys.path[:0] = sys.argv[1:4]
import numpy as np, torch, torch.distributed as dist
import oracle
from mlir_edsl.sharding import dense_rows
from gpu_util import max_err
rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
dev = torch.device("cuda", int(os.environ["LOCAL_RANK"]))
torch.cuda.set_device(dev)
dist.init_process_group("nccl", device_id=dev)
rows, N, K = 1000, 768, 512   # rows per rank; 3 slabs of 334/333/333
rng = np.random.default_rng(11)
X = rng.uniform(-1, 1, (world * rows, K)).astype(np.float32)
W = rng.uniform(-1, 1, (K, N)).astype(np.float32)
b = rng.uniform(-1, 1, N).astype(np.float32)
tX = torch.from_numpy(X[rank * rows:(rank + 1) * rows]).to(dev)
tW, tb = torch.from_numpy(W).to(dev), torch.from_numpy(b).to(dev)
ref = oracle.dense_f32(X, W, b, act=1)
for transport in ("ce", "nccl", "fused", "multimem"):
    for slabs in (1, 3, 3):  # the repeated call reuses the persistent IPC buffers
        Y = dense_rows(tX, tW, tb, 1, 0.0, gather=True, slabs=slabs, transport=transport)
        torch.cuda.synchronize()
        assert Y.shape == (world * rows, N)
        got = Y.cpu().numpy()
        assert max_err(got, ref) <= oracle.f32_bound(K, X, W), (transport, slabs)
# back-to-back gathered calls with no host synchronisation in between: the
# peer barriers on the stream order each call's stores against the peers'
# reads of the previous result (each result is copied out on the stream)
for transport in ("fused", "ce", "multimem"):
    outs = []
    for i in range(4):
        Xi = tX * (1.0 + 0.25 * i)
        Y = dense_rows(Xi, tW, tb, 1, 0.0, gather=True, slabs=2, transport=transport)
        outs.append(Y.clone())
    torch.cuda.synchronize()
    for i, Yi in enumerate(outs):
        Xs = (X * np.float32(1.0 + 0.25 * i)).astype(np.float32)
        assert max_err(Yi.cpu().numpy(), oracle.dense_f32(Xs, W, b, act=1)) <= \
            oracle.f32_bound(K, Xs, W), (transport, i)
loc = dense_rows(tX, tW, tb, 1, 0.0, gather=False).cpu().numpy()
assert loc.shape == (rows, N)
assert max_err(loc, got[rank * rows:(rank + 1) * rows]) <= oracle.f32_bound(K, X, W)
dist.destroy_process_group()
print("ok", rank)
"""


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_gather_rows_two_gpus_nccl(cuda):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    tests_dir = os.path.dirname(os.path.abspath(__file__))
    script = os.path.join(tests_dir, "_gather_two_gpus_script.py")
    with open(script, "w") as f:
        f.write(_SCRIPT)
    try:
        r = subprocess.run([sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
                            "--nproc-per-node", "2", "--master-addr", "127.0.0.1",
                            "--master-port", str(_port()), script, ROOT, PKG_PARENT, tests_dir],
                           capture_output=True, text=True, timeout=600,
                           env=dict(os.environ, NCCL_NVLS_ENABLE="0"))
    finally:
        os.remove(script)
    assert r.returncode == 0 and r.stdout.count("ok") == 2, (r.stdout[-2000:], r.stderr[-3000:])
