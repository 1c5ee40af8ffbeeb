"""Failure detection on the host (CPU, gloo ranks; no GPU is faulted or hung):

* a rank that announces its exit, and a rank that goes silent, are reported by the survivors'
  PeerMonitor before their next step;
* a rank that never reaches a barrier makes the others' bounded barrier raise;
* an engine whose peer died raises PeerFailureError from ``step`` instead of launching.
"""
import multiprocessing as mp
import os
import socket
import time


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _monitor_worker(rank, port, mode, q):
    from vllm_neuron_b200.parallel.health import PeerFailureError, PeerMonitor, make_store

    store = make_store("127.0.0.1", port, rank, 2)
    mon = PeerMonitor(store, rank, 2, interval_s=0.1, timeout_s=1.0)
    # both ranks are up
    deadline = time.time() + 10
    while not store.check([f"b200/hb/{1 - rank}"]) and time.time() < deadline:
        time.sleep(0.05)
    store.set(f"ready/{rank}", "1")
    store.wait([f"ready/{1 - rank}"])
    if rank == 1:
        if mode == "exit":
            mon.stop(announce_exit=True)
            q.put((1, "left"))
            store.wait(["done"])
            return
        mon.stop(announce_exit=False)  # silent: alive but no more heartbeats
        q.put((1, "silent"))
        store.wait(["done"])
        return
    t0 = time.time()
    try:
        while time.time() - t0 < 15:
            mon.check()
            time.sleep(0.05)
        q.put((0, "not detected"))
    except PeerFailureError as e:
        q.put((0, ("detected", e.rank, str(e), time.time() - t0)))
    store.set("done", "1")


def _run_pair(target, *args):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=target, args=(r, port) + args + (q,)) for r in range(2)]
    for p in ps:
        p.start()
    res = dict(q.get(timeout=60) for _ in ps)
    for p in ps:
        p.join(timeout=30)
    return res


def test_peer_exit_detected():
    res = _run_pair(_monitor_worker, "exit")
    assert res[0][0] == "detected" and res[0][1] == 1 and "exit" in res[0][2]
    assert res[0][3] < 5


def test_silent_peer_detected_by_heartbeat_timeout():
    res = _run_pair(_monitor_worker, "silent")
    assert res[0][0] == "detected" and "heartbeat" in res[0][2]
    assert res[0][3] < 8


def _barrier_worker(rank, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch.distributed as dist

    from vllm_neuron_b200.parallel import state as ps

    dist.init_process_group("gloo", rank=rank, world_size=2)
    ps.initialize_parallel_state(ps.ParallelConfig(world_size=2, tensor_parallel_size=2))
    if rank == 1:
        q.put((1, "skipped"))
        time.sleep(6)  # never joins the barrier
        return
    t0 = time.time()
    try:
        ps.world_barrier(timeout_s=2.0)
        q.put((0, "no error"))
    except Exception as e:
        q.put((0, ("raised", type(e).__name__, time.time() - t0)))


def test_barrier_times_out_when_a_rank_never_joins():
    res = _run_pair(_barrier_worker)
    assert res[0][0] == "raised" and res[0][2] < 10


def _engine_worker(rank, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE="2",
                      LOCAL_RANK=str(rank), VLLM_B200_HEARTBEAT_TIMEOUT="2", VLLM_B200_HEARTBEAT_INTERVAL="0.1")
    import torch

    torch.set_num_threads(1)
    from tests._tiny import random_prompts, tiny_llama_checkpoint
    from vllm_neuron_b200.engine.sampling_params import SamplingParams
    from vllm_neuron_b200.entrypoints import LLM
    from vllm_neuron_b200.parallel.health import PeerFailureError

    ckpt, _ = tiny_llama_checkpoint()
    llm = LLM(ckpt, tensor_parallel_size=2, device="cpu", max_num_seqs=4, max_model_len=128,
              num_gpu_blocks=64, max_num_batched_tokens=64)
    sp = SamplingParams(temperature=0, max_tokens=4, ignore_eos=True)
    llm.generate(random_prompts(n=2, length=10, seed=1), sp)  # both ranks serve one batch
    if rank == 1:
        llm.engine.monitor.stop(announce_exit=True)  # leaves between steps
        q.put((1, "left"))
        time.sleep(3)
        return
    # the peer leaves between steps; this rank's next step must notice it on the host
    llm.engine.monitor.store.wait(["b200/exit/1"])
    try:
        llm.generate(random_prompts(n=2, length=10, seed=2), sp)
        q.put((0, "no error"))
    except PeerFailureError as e:
        q.put((0, ("detected", e.rank)))
    except Exception as e:  # pragma: no cover
        q.put((0, ("other", repr(e))))


def test_engine_step_reports_dead_peer():
    res = _run_pair(_engine_worker)
    assert res[0] == ("detected", 1), res
