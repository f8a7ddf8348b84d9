"""Host-side pieces of the benchmark's reference arm (no GPU, no vLLM engine):
the N=1 unavailability line, the K4/V2 profile being accepted by the
reference's own adapter, and the store barrier used to sequence requests."""
import json
import os
import subprocess
import sys

import pytest
import torch.multiprocessing as mp

from kvserve_b200.baselines import reference_arm as ra

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_one_gpu_prints_unavailable_line():
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference"],
                         capture_output=True, text=True, timeout=300, cwd=ROOT)
    assert out.returncode == 0
    line = json.loads(out.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference" and "unavailable" in line


@pytest.mark.skipif(not os.path.isdir(os.path.join(ra.REF_DIR, "kvserve_v1")), reason="reference not installed")
def test_k4v2_profile_accepted_by_reference_adapter():
    sys.path.insert(0, ra.REF_DIR)
    try:
        from kvserve_v1.compression.manager import KVCompressionAdapter
        KVCompressionAdapter(ra.reference_profile("k4v2"), 8, 128)
    finally:
        sys.path.remove(ra.REF_DIR)
    assert ra.reference_profile("raw") is None


def _barrier_worker(rank, port, q):
    import time
    bar = ra._Barrier("127.0.0.1", port, rank, 2, timeout_s=60)
    order = []
    for i in range(3):
        bar.wait()
        if rank == 0:
            time.sleep(0.05)
            bar.set(f"done{i}", str(i))
        else:
            order.append(int(bar.get(f"done{i}")))
    q.put((rank, order))


def test_store_barrier_sequences_two_processes():
    import datetime
    import socket
    import torch.distributed as dist
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    master = dist.TCPStore("127.0.0.1", port, is_master=True, wait_for_workers=False,
                           timeout=datetime.timedelta(seconds=60))
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_barrier_worker, args=(r, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = dict(q.get(timeout=120) for _ in ps)
    for p in ps:
        p.join(30)
    assert res[1] == [0, 1, 2]
    del master


def test_vllm_compat_view_gives_reference_shape_over_real_cache():
    """The adapter hands the reference's consumer what the older vLLM API
    gave it (virtual_engine 0, per-virtual-engine cache list) while the
    tensor it writes is vLLM's own cache tensor."""
    import types
    import torch
    from kvserve_b200.baselines import vllm_compat as vc
    cache = torch.zeros(2, 3, 4)
    layer = types.SimpleNamespace(kv_cache=cache, layer_name="l0")
    real_ctx = types.SimpleNamespace(no_compile_layers={"l0": layer}, attn_metadata={"x": 1})
    mod = types.SimpleNamespace(get_forward_context=lambda: real_ctx)
    assert vc._wrap_module(mod) and not vc._wrap_module(mod)   # wrapped once
    fc = mod.get_forward_context()
    assert fc.virtual_engine == 0 and fc.attn_metadata == {"x": 1}
    got = fc.no_compile_layers.get("l0")
    kv = got.kv_cache[fc.virtual_engine]          # the reference's access pattern
    assert kv is cache and got.layer_name == "l0"
    kv[0].fill_(1.0)
    assert cache[0].sum() == 12
    assert fc.no_compile_layers.get("missing") is None and list(fc.no_compile_layers) == ["l0"]


def test_vllm_compat_entry_point_is_discoverable(tmp_path):
    from kvserve_b200.baselines import vllm_compat as vc
    d = vc.install_entry_point(str(tmp_path))
    code = ("from importlib.metadata import entry_points;"
            "print([e.value for e in entry_points(group='vllm.general_plugins') if e.name == %r])" % vc.PLUGIN_NAME)
    env = dict(os.environ, PYTHONPATH=os.pathsep.join([d, ROOT]))
    out = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, env=env, timeout=120)
    assert "kvserve_b200.baselines.vllm_compat:register" in out.stdout, out.stderr


def _failing_worker(rank, port, q):
    bar = ra._Barrier("127.0.0.1", port, rank, 2, timeout_s=60)
    try:
        if rank == 1:
            ra._role_call(bar, "consumer request", lambda: 1 / 0)
        bar.wait()                     # rank 0 must not wait forever for rank 1
        q.put((rank, "passed"))
    except ra.ArmFailure as exc:
        q.put((rank, str(exc)))
    bar.wait("final", allow_failed=True)


def test_store_barrier_propagates_a_role_failure():
    import datetime
    import socket
    import torch.distributed as dist
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    master = dist.TCPStore("127.0.0.1", port, is_master=True, wait_for_workers=False,
                           timeout=datetime.timedelta(seconds=60))
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_failing_worker, args=(r, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = dict(q.get(timeout=120) for _ in ps)
    for p in ps:
        p.join(30)
    assert "ZeroDivisionError" in res[0] and "ZeroDivisionError" in res[1]
    del master
