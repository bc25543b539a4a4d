"""Host logic of the multi-GPU path on CPU: event-balanced sample sharding, the gather of the
logits back into input order (gloo ranks standing in for NCCL ones), and a rank that fails
before the gather, which the surviving rank must see as an error rather than a hang."""
import multiprocessing as mp
import os
import socket
import time
import traceback

import numpy as np
import pytest

import salt_b200 as S
from salt_b200.sharding import balanced_shards, take_shard, unshard


def test_balanced_shards_cover_every_sample_once_and_balance_events():
    rng = np.random.default_rng(0)
    n = np.exp(rng.uniform(np.log(2000), np.log(20000), 1001)).astype(np.int64)
    for world in (1, 2, 3, 8):
        sh = balanced_shards(n, world)
        flat = sh.index.reshape(-1)
        real = flat[flat != sh.pad_index]
        assert sorted(real.tolist()) == list(range(len(n)))
        assert sh.counts.sum() == len(n) and sh.counts.max() <= sh.per_rank
        assert sh.events.sum() == n.sum()
        # greedy LPT: the heaviest and lightest ranks differ by at most the largest sample
        assert sh.events.max() - sh.events.min() <= n.max()
        for r in range(world):  # input order inside a shard
            idx = sh.of(r)[: sh.counts[r]]
            assert np.all(np.diff(idx) > 0)
        rows = np.arange(len(n))[:, None] * np.array([[1, -1]])
        gathered = np.concatenate([take_shard([rows], sh, r)[0] for r in range(world)])
        np.testing.assert_array_equal(unshard(gathered, sh), rows)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


class _GlooComm:
    """The communicator interface gather_rows takes (world, all_gather), over torch's gloo
    process group on host arrays: the CPU stand-in for comm.NcclComm."""

    def __init__(self, world):
        self.world = world

    def all_gather(self, send, recv):
        import torch
        import torch.distributed as dist
        dist.all_gather_into_tensor(torch.from_numpy(recv), torch.from_numpy(send))


def _rank_main(rank, world, port, mode, q):
    """One gloo rank: run the CPU oracle network on this rank's shard, gather the logits."""
    try:
        import datetime
        import torch
        import torch.distributed as dist
        import oracle as O
        from salt_b200.sharding import balanced_shards, gather_rows, take_shard, unshard
        from _cases import make_events, make_params
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=10))
        rng = np.random.default_rng(7)   # the same global batch on every rank
        net = S.Network.build((2, 8, 8), [
            S.conv(4, k=3, s=2, p=1, init_k=5.0, max_queue_len=64, max_out_spikes=256),
            S.fc(6, init_k=5.0, v_th=1e9, max_out_spikes=1)])
        params = [make_params(l, rng, vth=(40, 90), f_a=8, fires=i == 0)
                  for i, l in enumerate(net.layers)]
        times, src, nr = make_events(rng, 9, 60, 128, t_max=40)
        sh = balanced_shards(nr, world)
        if mode == "fail" and rank == 1:
            raise RuntimeError("planted failure on rank 1 before the gather")
        t, s, n = take_shard([times, src, nr], sh, rank)
        n = np.where(sh.of(rank) == sh.pad_index, 0, n)
        logits, _, _ = O.network_batch(net.layers, params, t, s, n, threads=1)
        full = gather_rows(np.ascontiguousarray(logits, dtype=np.int32), _GlooComm(world))
        got = unshard(full, sh)
        ref, _, _ = O.network_batch(net.layers, params, times, src, nr, threads=1)
        q.put((rank, "ok", bool(np.array_equal(got, ref))))
        dist.destroy_process_group()
    except Exception as e:  # noqa: BLE001 - reported to the test
        q.put((rank, "error", f"{type(e).__name__}: {e}\n{traceback.format_exc()[-400:]}"))


def _run_ranks(world, mode, limit=60.0):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    results, t0 = {}, time.time()
    while len(results) < world and time.time() - t0 < limit:
        try:
            r, status, detail = q.get(timeout=1.0)
            results[r] = (status, detail)
        except Exception:  # noqa: BLE001 - queue.Empty
            pass
    for p in procs:
        p.join(timeout=5)
        if p.is_alive():
            p.kill()
    return results


def test_two_gloo_ranks_gather_logits_in_input_order():
    res = _run_ranks(2, "ok")
    assert res.get(0, ("missing",))[0] == "ok", res
    assert res.get(1, ("missing",))[0] == "ok", res
    assert res[0][1] is True and res[1][1] is True


def test_a_failed_rank_ends_the_other_ranks_gather_with_an_error():
    t0 = time.time()
    res = _run_ranks(2, "fail")
    assert res.get(1, ("missing",))[0] == "error" and "planted failure" in res[1][1]
    assert res.get(0, ("missing",))[0] == "error", res   # an error, not a hang
    assert time.time() - t0 < 60
