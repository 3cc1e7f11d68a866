"""Allreduce kernels on the GPU.

* Single GPU: the bounded device wait. A 2-rank context whose "peer" is a
  local buffer that never signals: the kernel's wait must give up after the
  timeout, record (code, block, peer, phase) in host-mapped memory and return;
  the host raises MailboxError and the CUDA context stays usable. No GPU
  fault, no trap, one kernel waiting on a flag nothing sets.
* 2+ GPUs: tests/mp_allreduce_worker.py under torchrun (one process per GPU).
"""
import os
import subprocess
import sys

import pytest
import torch

from conftest import ROOT, free_port, sub

pytestmark = pytest.mark.gpu


def test_device_wait_times_out_and_reports():
    C = sub("_ext").cuda_ext()
    half = 1 << 20
    size = C.SIG_BYTES + 2 * half
    mine = torch.zeros(size, dtype=torch.uint8, device="cuda")
    fake_peer = torch.zeros(size, dtype=torch.uint8, device="cuda")  # never signals
    state = torch.zeros(C.STATE_WORDS, dtype=torch.int32, device="cuda")
    status = C.host_mapped_alloc(4 * C.STATUS_WORDS)
    try:
        ar = C.ArComm(0, 2, [mine.data_ptr(), fake_peer.data_ptr()], 0, state.data_ptr(), status.dev, status.host,
                      half, 0, 50_000_000)  # 50 ms bound
        x = torch.ones(4096, dtype=torch.bfloat16, device="cuda")
        out = torch.empty_like(x)
        ar.allreduce(x.data_ptr(), out.data_ptr(), x.numel() * 2, 2, 1, 4, 0)
        torch.cuda.synchronize()
        st = ar.status()
        assert st[0] == 3, st            # barrier wait gave up
        assert st[2] == 1 and st[3] == 0  # waiting for rank 1 in phase 0
        assert int(state[2].item()) == 3  # device-side sticky copy
        # later calls early-exit on the sticky error (no second wait)
        ar.allreduce(x.data_ptr(), out.data_ptr(), x.numel() * 2, 2, 1, 4, 0)
        torch.cuda.synchronize()
        # the context is still healthy
        y = torch.arange(10, device="cuda").sum().item()
        assert y == 45
    finally:
        C.host_mapped_free(status.host)


def _ngpus():
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


@pytest.mark.multigpu
@pytest.mark.skipif(_ngpus() < 2, reason="needs 2+ GPUs")
def test_multi_gpu_allreduce_suite():
    n = min(_ngpus(), 8)
    env = dict(os.environ)
    env["PYTHONPATH"] = ROOT + os.pathsep + env.get("PYTHONPATH", "")
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={n}", "--master-addr=127.0.0.1", f"--master-port={free_port()}",
           os.path.join(ROOT, "tests", "mp_allreduce_worker.py")]
    p = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=700)
    out = p.stdout + "\n" + p.stderr
    err_at = out.find("WORKER-ERROR")
    detail = out[err_at:err_at + 6000] if err_at >= 0 else out[-4000:]
    assert p.returncode == 0, detail
    assert "ALLREDUCE-SUITE-PASS" in p.stdout, detail
