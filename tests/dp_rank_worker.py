"""One rank of the two-process data-parallel GPU tests (tests/test_dp_gpu.py),
launched by torchrun exactly as bench.py's ranks are: a gloo process group
for the host side, the PJRT client on GPU LOCAL_RANK with node_id / num_nodes
and the key-value callbacks over the process group's store (rank 0 publishes
the NCCL unique id there), and the `num_replicas=2` step on this rank's half
of the batch.

    python -m torch.distributed.run --nproc-per-node=2 ... dp_rank_worker.py OUT KIND

KIND is "mlp" (configs[2], SGD step) or "transformer" (configs[3]
architecture at reduced size, gradients).  Writes OUT/rank<r>.npz with the
outputs, or OUT/rank<r>.err with "<code> <message>" when Execute raises a
PJRT error; OUT/rank<r>.stage names the last stage reached.

KIND "leave": both ranks run one data-parallel step; then rank 1 leaves (it
exits between steps, with nothing of its own in flight) and rank 0 runs the
next step, whose all-reduce can never complete.  The plugin's NCCL watchdog
must end it with an error (B200_NCCL_TIMEOUT_MS), and the step after that must
be refused at once.  Rank 0 writes OUT/leave.txt: the codes it saw."""
import os
import sys
from datetime import timedelta

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
sys.path[:0] = [HERE, ROOT, os.path.join(ROOT, "jax-mlx-plugin_b200")]


def main():
    out, kind = sys.argv[1], sys.argv[2]
    rank = int(os.environ["RANK"])
    local = int(os.environ["LOCAL_RANK"])

    def stage(s):
        with open(os.path.join(out, f"rank{rank}.stage"), "w") as f:
            f.write(s)

    import faulthandler
    fault_log = open(os.path.join(out, f"rank{rank}.fault"), "w")
    faulthandler.enable(file=fault_log, all_threads=True)

    stage("init")
    import torch
    import torch.distributed as dist
    torch.cuda.set_device(local)
    dist.init_process_group("gloo", timeout=timedelta(seconds=120))
    store = dist.distributed_c10d._get_default_store()

    class KV:
        def set(self, k, v):
            store.set(k, v)

        def get(self, k):
            return bytes(store.get(k))

    from jax_b200 import pjrt, programs
    from test_dp_gpu import TR_SMALL, _kink_safe_mlp, _to_np, _tr_inputs
    stage("client")
    client = pjrt.Client({"visible_devices": [local], "node_id": rank, "num_nodes": 2}, kv=KV())
    dev = client.addressable_devices[0]
    stage("compile")
    if kind == "leave":
        return leave(rank, out, stage, client, dev, store, dist)
    if kind == "mlp":
        dims = (784, 1024, 1024, 1024, 10)
        params, x, lab = _kink_safe_mlp(np.random.default_rng(53), dims, 1024)
        sl = slice(512 * rank, 512 * (rank + 1))
        exe = client.compile(programs.mlp_step(batch=512, dims=dims, num_replicas=2))
        arrays = params + [x[sl], lab[sl]]
        bf16 = 0
    else:
        names, params, zeros, count, tok, tgt = _tr_inputs(TR_SMALL, 54)
        sl = slice(2 * rank, 2 * (rank + 1))
        exe = client.compile(programs.transformer_step(**dict(TR_SMALL, batch=2), num_replicas=2,
                                                       emit="grads"))
        arrays = [pjrt.to_bf16_bits(p) for p in params] + zeros + zeros + [count, tok[sl], tgt[sl]]
        bf16 = len(params)
    args = [client.buffer_from_numpy(a, device=dev, bf16=i < bf16) for i, a in enumerate(arrays)]
    stage("execute")
    outs = None
    try:
        outs = exe.execute([args])[0]
        stage("read")
        res = [_to_np(o) for o in outs]
        np.savez(os.path.join(out, f"rank{rank}.npz"), *res)
    except pjrt.PjrtError as e:
        with open(os.path.join(out, f"rank{rank}.err"), "w") as f:
            f.write(f"{e.code} {e}")
    stage("barrier")
    dist.barrier()
    outs = None  # every buffer and executable goes before the client
    del args, exe, outs
    stage("client_destroy")
    client.destroy()
    stage("done")
    dist.destroy_process_group()


def leave(rank, out, stage, client, dev, store, dist):
    import time
    from jax_b200 import pjrt, programs
    dims = (64, 128, 10)
    rng = np.random.default_rng(55)
    params = [(rng.standard_normal(s) * 0.1).astype(np.float32)
              for s in ((64, 128), (128,), (128, 10), (10,))]
    x = rng.random((16, 64)).astype(np.float32)
    lab = rng.integers(0, 10, 16).astype(np.int32)
    exe = client.compile(programs.mlp_step(batch=8, dims=dims, num_replicas=2))
    args = [client.buffer_from_numpy(a, device=dev) for a in params + [x[8 * rank:8 * rank + 8],
                                                                       lab[8 * rank:8 * rank + 8]]]
    stage("step1")
    loss1 = float(exe.execute([args])[0][0].to_numpy())
    if rank == 1:
        stage("left")
        store.set("b200_test/rank1_left", b"1")
        dist.destroy_process_group()
        os._exit(0)  # leaves between steps: no kernel or collective of its own in flight
    store.wait(["b200_test/rank1_left"])
    time.sleep(2.0)
    res = [f"step1 {loss1:.6f}"]
    stage("step2")
    t0 = time.time()
    try:
        exe.execute([args])[0][0].to_numpy()
        res.append("step2 ok")
    except pjrt.PjrtError as e:
        res.append(f"step2 {e.code} {time.time() - t0:.1f}s {e}")
    stage("step3")
    try:
        exe.execute([args])[0][0].to_numpy()
        res.append("step3 ok")
    except pjrt.PjrtError as e:
        res.append(f"step3 {e.code} {e}")
    with open(os.path.join(out, "leave.txt"), "w") as f:
        f.write("\n".join(res) + "\n")
    stage("done")
    os._exit(0)  # rank 1 is gone: no process-group teardown with it


if __name__ == "__main__":
    main()
