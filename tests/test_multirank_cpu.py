"""CPU, world size 2 over gloo: the host side of the one-process-per-GPU path.

* NCCL bootstrap: rank 0 of a multi-process job publishes the NCCL unique id
  through the client's PJRT key-value put callback and the other ranks read it
  through the get callback (`csrc/host/pjrt.cc:comms_for`).  Here both
  callbacks run over a torch.distributed store in two real processes, as
  `bench.py` wires them, with a 128-byte id that holds zero bytes.
* Data parallelism: each rank evaluates the `num_replicas=2` training step on
  its half of the batch (the slice `bench.py` gives it) with the all_reduce
  summed across the processes; both ranks end with the full-batch step.
* `bench.py --impl reference` under torchrun: rank 0 alone prints the line.
No GPU and no plugin compute call is involved."""
import ctypes as C
import json
import multiprocessing as mp
import os
import socket
import subprocess
import sys
from datetime import timedelta

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
WORLD = 2
UID_KEY = "b200/nccl_uid/2"


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, port):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=WORLD, timeout=timedelta(seconds=60))
    return dist


class _StoreKV:
    """The adapter bench.py hands the client: str keys, bytes values."""

    def __init__(self, store):
        self.store = store

    def set(self, k, v):
        self.store.set(k, v)

    def get(self, k):
        return bytes(self.store.get(k))


def _uid():
    rng = np.random.default_rng(7)
    b = bytearray(rng.integers(0, 256, 128, dtype=np.uint8).tobytes())
    b[0] = b[17] = b[127] = 0
    return bytes(b)


def _kv_worker(rank, port, out):
    dist = _init(rank, port)
    from jax_b200 import pjrt
    get_cb, put_cb, keep = pjrt.kv_callbacks(_StoreKV(dist.distributed_c10d._get_default_store()))
    key = UID_KEY.encode()
    if rank == 0:
        val = _uid()
        a = pjrt.KVPutArgs()
        a.struct_size = C.sizeof(a)
        a.key, a.key_size = key, len(key)
        vbuf = C.create_string_buffer(val, len(val))
        a.value, a.value_size = C.addressof(vbuf), len(val)
        assert put_cb(C.pointer(a)) is None
        got = val
    else:
        a = pjrt.KVGetArgs()
        a.struct_size = C.sizeof(a)
        a.key, a.key_size = key, len(key)
        a.timeout_in_ms = 30000
        assert get_cb(C.pointer(a)) is None
        got = C.string_at(a.value, a.value_size)
        # the plugin frees the value through the deleter it was given
        assert len(keep[-1]) == 1
        pjrt.VALUE_DELETER(a.value_deleter_callback)(a.value)
        assert len(keep[-1]) == 0
    dist.barrier()
    with open(os.path.join(out, f"uid{rank}.bin"), "wb") as f:
        f.write(got)
    dist.destroy_process_group()


def _mlp_inputs(dims, batch):
    rng = np.random.default_rng(21)
    params = []
    for i in range(len(dims) - 1):
        params.append((rng.standard_normal((dims[i], dims[i + 1])) * 0.3).astype(np.float32))
        params.append((rng.standard_normal(dims[i + 1]) * 0.1).astype(np.float32))
    x = rng.random((batch, dims[0])).astype(np.float32)
    lab = rng.integers(0, dims[-1], batch).astype(np.int32)
    return params, x, lab


DIMS, BATCH = (20, 16, 16, 5), 8


def _dp_worker(rank, port, out):
    dist = _init(rank, port)
    import torch
    from jax_b200 import programs
    from oracle import hlo_interp

    def process_sum(a):
        t = torch.from_numpy(np.ascontiguousarray(a, np.float64))
        dist.all_reduce(t)
        return t.numpy()

    params, x, lab = _mlp_inputs(DIMS, BATCH)
    per = BATCH // WORLD
    sl = slice(rank * per, (rank + 1) * per)  # bench.py's shard of the global batch
    text = programs.mlp_step(batch=per, dims=DIMS, num_replicas=WORLD)
    outs = hlo_interp.run(text, [params + [x[sl], lab[sl]]], process_sum=process_sum)[0]
    np.savez(os.path.join(out, f"dp{rank}.npz"), *outs)
    dist.destroy_process_group()


def _spawn(fn, out):
    ctx = mp.get_context("spawn")
    port = _free_port()
    ps = [ctx.Process(target=fn, args=(r, port, out)) for r in range(WORLD)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(180)
    for p in ps:
        if p.is_alive():
            p.kill()
            p.join()
    assert [p.exitcode for p in ps] == [0] * WORLD


def test_nccl_id_crosses_processes_through_kv_callbacks(tmp_path):
    _spawn(_kv_worker, str(tmp_path))
    got = [(tmp_path / f"uid{r}.bin").read_bytes() for r in range(WORLD)]
    assert got[0] == got[1] == _uid() and len(got[1]) == 128


@pytest.mark.filterwarnings("ignore::pytest.PytestUnraisableExceptionWarning")
def test_failed_store_get_leaves_value_unset():
    """A store whose get raises (rank 0 gone, store timeout) cannot hand the
    plugin an error object from Python; the callback then leaves the value
    unset, which the plugin reports as a failed KV get naming the key."""
    from jax_b200 import pjrt

    class Broken:
        def set(self, k, v):
            pass

        def get(self, k):
            raise TimeoutError(k)

    get_cb, _, _ = pjrt.kv_callbacks(Broken())
    a = pjrt.KVGetArgs()
    a.struct_size = C.sizeof(a)
    key = UID_KEY.encode()
    a.key, a.key_size = key, len(key)
    get_cb(C.pointer(a))  # ctypes reports the exception and returns null
    assert not a.value and a.value_size == 0


def test_data_parallel_step_across_processes_equals_full_batch(tmp_path):
    from jax_b200 import programs
    from oracle import hlo_interp
    _spawn(_dp_worker, str(tmp_path))
    params, x, lab = _mlp_inputs(DIMS, BATCH)
    full = hlo_interp.run(programs.mlp_step(batch=BATCH, dims=DIMS), [params + [x, lab]])[0]
    for r in range(WORLD):
        z = np.load(tmp_path / f"dp{r}.npz")
        got = [z[f"arr_{i}"] for i in range(len(z.files))]
        assert len(got) == len(full)
        for a, b in zip(got, full):
            np.testing.assert_allclose(a, b, rtol=1e-6, atol=1e-7)


def test_bench_reference_arm_prints_once_under_torchrun():
    port = _free_port()
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={WORLD}",
           "--master-addr", "127.0.0.1", "--master-port", str(port), "bench.py", "--impl", "reference",
           "--gpus", str(WORLD), "--steps", "1", "--warmup", "3"]
    r = subprocess.run(cmd, cwd=ROOT, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [json.loads(l) for l in r.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    line = lines[0]
    assert line["impl"] == "reference" and line["n_gpus"] == WORLD and line["value"] > 0
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["cpu_baseline"]["cores"] >= 1


class _DictStore:
    def __init__(self):
        self.d = {}

    def set(self, k, v):
        self.d[k] = bytes(v)

    def get(self, k):
        if k not in self.d:
            raise TimeoutError(f"key {k} not set within the store's timeout")
        return self.d[k]


def test_kv_exchange_round_trip_through_plugin():
    """The plugin's NCCL-id exchange (rank 0 puts, others get) through the
    Python callbacks: 128 bytes with zeros arrive unchanged."""
    from jax_b200 import pjrt
    st = _DictStore()
    uid = _uid()
    assert pjrt.kv_exchange(st, 0, UID_KEY, uid) == uid
    assert st.d[UID_KEY] == uid
    assert pjrt.kv_exchange(st, 1, UID_KEY) == uid


def test_kv_store_errors_become_pjrt_errors_with_their_code():
    """jaxlib's KV wrappers report a failed store call by building the error
    through args->callback_error; the plugin must hand them a constructor and
    turn the returned object into a PJRT error (here DEADLINE_EXCEEDED for a
    get that timed out, UNKNOWN for a put that raised)."""
    from jax_b200 import pjrt

    class PutFails(_DictStore):
        def set(self, k, v):
            raise ConnectionError("store gone")

    with pytest.raises(pjrt.PjrtError) as e:
        pjrt.kv_exchange(_DictStore(), 1, UID_KEY)
    assert e.value.code == 4 and UID_KEY in str(e.value) and "TimeoutError" in str(e.value)
    with pytest.raises(pjrt.PjrtError) as e:
        pjrt.kv_exchange(PutFails(), 0, UID_KEY, b"x")
    assert e.value.code == 2 and "store gone" in str(e.value)


def test_raw_kv_callback_error_keeps_its_code():
    """A C-level get callback, as jaxlib writes it: on failure it returns
    (*args->callback_error)(NOT_FOUND, msg, n) and the plugin reports code 5."""
    from jax_b200 import pjrt
    lib = pjrt.api().lib
    msg = b"no such key"

    def raw_get(args):
        a = args.contents
        assert a.callback_error, "plugin passed no callback_error"
        make = C.cast(a.callback_error, C.POINTER(pjrt.CALLBACK_ERROR))[0]
        return make(5, msg, len(msg))

    cb = pjrt.KV_GET_CB(raw_get)
    fn = lib.b200_pjrt_kv_exchange
    fn.argtypes = [C.c_void_p] * 4 + [C.c_int, C.c_char_p, C.c_size_t, C.c_char_p, C.c_size_t,
                                      C.POINTER(C.c_void_p), C.POINTER(C.c_size_t)]
    out, n = C.c_void_p(), C.c_size_t(0)
    rc = fn(C.cast(cb, C.c_void_p), None, None, None, 1, b"k", 1, None, 0, C.byref(out), C.byref(n))
    text = C.string_at(out.value, n.value).decode()
    lib.b200_pjrt_free(out)
    assert rc == 5 and "no such key" in text
