"""GPU-driven NVLink channels between two processes: several messages,
some larger than a ring slot (sent in pieces), checked byte for byte."""
import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

_CHILD = r"""
import os, json, torch, torch.distributed as dist
from datetime import timedelta
from connex_b200.parallel.p2pchan import ChanLinks
rank = int(os.environ["RANK"]); dev = torch.device("cuda", int(os.environ["LOCAL_RANK"]))
torch.cuda.set_device(dev)
dist.init_process_group("gloo", timeout=timedelta(seconds=60))
store = dist.distributed_c10d._get_default_store()
ch = ChanLinks(dist.PrefixStore("t/", store), f"e{rank}", dev, slots=2, slot_bytes=1 << 20)
ok = True
shapes = [(8, 64), (1024, 1024), (3, 4096), (2048, 1024)]       # 1 KB ... 4 MB (4 pieces)
for i, s in enumerate(shapes):
    g = torch.Generator(device=dev); g.manual_seed(i)
    x = torch.randn(*s, device=dev, generator=g).bfloat16()
    y = torch.randn(s[0], 8, device=dev, generator=g)
    if rank == 0:
        ch.open_tx("e1").send([x, y])
    else:
        a, b = torch.empty_like(x), torch.empty_like(y)
        rx = ch.open_rx("e0")
        rx.recv([a, b])
        torch.cuda.current_stream(dev).wait_event(rx.done_event())
        torch.cuda.synchronize(dev)
        ok &= bool(torch.equal(a, x) and torch.equal(b, y))
torch.cuda.synchronize(dev)
ch.check()
res = [None, None]
dist.all_gather_object(res, ok)
if rank == 0:
    print(json.dumps(res))
dist.barrier()
ch.close()
dist.destroy_process_group()
"""


def test_channel_two_gpus(tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    script = tmp_path / "child.py"
    script.write_text(_CHILD)
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    r = subprocess.run(["timeout", "-k", "10", "120", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
                        "--nproc-per-node", "2", "--master-addr", "127.0.0.1", "--master-port", "29651", str(script)],
                       capture_output=True, text=True, env=dict(os.environ, PYTHONPATH=root), cwd=root)
    assert r.returncode == 0, r.stderr[-3000:]
    assert "[true, true]" in r.stdout


def test_cancelled_channel_launch_returns_at_once():
    """A launch waiting on a counter that nothing will raise (its peer died)
    returns as soon as the host raises the link's abort word, long before its
    timeout, with status peer-abort and nothing copied; a launch queued after
    the abort does not wait at all."""
    import time
    from connex_b200 import ops
    dev = torch.device("cuda", 0)
    status = ops.new_status(dev)
    flag = torch.zeros(4, dtype=torch.int32, device=dev)          # never raised
    src = torch.randn(4096, device=dev)
    dst = torch.zeros_like(src)
    abort = torch.zeros(4, dtype=torch.int32).pin_memory()
    nbytes = src.numel() * 4
    torch.cuda.synchronize()
    t0 = time.monotonic()
    ops._C.chan_copy([src.data_ptr()], [dst.data_ptr()], [nbytes], flag.data_ptr(), 1, int(20e9), 0, 0, 0, 0, 1,
                     status, abort.data_ptr())
    time.sleep(0.3)
    abort[0] = 1
    torch.cuda.synchronize()
    assert time.monotonic() - t0 < 5.0
    assert int(status.item()) == 3 and int(dst.abs().sum().item()) == 0
    status.zero_()
    ops._C.chan_copy([src.data_ptr()], [dst.data_ptr()], [nbytes], 0, 0, int(20e9), 0, 0, 0, 0, 1, status,
                     abort.data_ptr())
    torch.cuda.synchronize()
    assert int(status.item()) == 3 and int(dst.abs().sum().item()) == 0
    # without an abort word the same launch copies
    status.zero_()
    ops._C.chan_copy([src.data_ptr()], [dst.data_ptr()], [nbytes], 0, 0, int(20e9), 0, 0, 0, 0, 1, status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0 and torch.equal(dst, src)
