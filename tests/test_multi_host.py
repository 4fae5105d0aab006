"""Host-side logic of the batch-sharded multi-GPU path, on CPU with gloo
(world size 2): shard ranges tile the batch, each rank's shard computed from
its own regenerated inputs equals the same rows of the 1-process result, and
the gathered output equals the full output bit for bit."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from fmha_b200.multi import make_shard, shard_rows


@pytest.mark.parametrize("batch,world", [(30720, 8), (7, 2), (10, 3), (1, 4)])
def test_shards_tile_the_batch(batch, world):
    spans = [shard_rows(batch, world, r) for r in range(world)]
    assert spans[0][0] == 0 and spans[-1][1] == batch
    for (a, b), (c, _) in zip(spans, spans[1:]):
        assert b == c and b >= a
    assert max(b - a for a, b in spans) - min(b - a for a, b in spans) <= 1
    with pytest.raises(ValueError):
        shard_rows(batch, world, world)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


SHAPE = (13, 32, 16, 5, 128)  # batch, hq, hkv, s, d (ragged shards: 7 + 6 rows)


def _worker(rank, world, port, outdir, shape=SHAPE):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from fmha_b200.multi import gather_output
    from oracle import oracle as O
    b, hq, hkv, s, d = shape
    sh = make_shard(b, hq, hkv, s, d, world, rank)
    q, k, v = O.make_inputs_bhsd(sh.rows, hq, hkv, s, d, seed=9, batch_offset=sh.row0)
    _, o16 = O.decode_bhsd(q, k, v, sh.rows, hq, hkv, s, d, want_f32=False)
    full = gather_output(torch.from_numpy(o16.view(np.int16)), sh)
    t = torch.tensor([float(rank + 1)])
    dist.all_reduce(t, op=dist.ReduceOp.MAX)  # max-over-ranks timing reduction
    np.save(os.path.join(outdir, f"r{rank}.npy"), full.numpy())
    np.save(os.path.join(outdir, f"m{rank}.npy"), t.numpy())
    dist.destroy_process_group()


@pytest.mark.parametrize("shape", [SHAPE, (12, 16, 16, 3, 128)], ids=["ragged", "equal"])
def test_gloo_two_rank_shards_equal_single_process(tmp_path, oracle, shape):
    """Ragged shards take the padded all-gather, equal shards the single
    all_gather_into_tensor; both must give the 1-process output."""
    world = 2
    mp.spawn(_worker, args=(world, _free_port(), str(tmp_path), shape), nprocs=world, join=True)
    b, hq, hkv, s, d = shape
    q, k, v = oracle.make_inputs_bhsd(b, hq, hkv, s, d, seed=9)
    _, ref = oracle.decode_bhsd(q, k, v, b, hq, hkv, s, d, want_f32=False)
    for r in range(world):
        got = np.load(tmp_path / f"r{r}.npy").view(np.uint16)
        assert np.array_equal(got, ref)
        assert float(np.load(tmp_path / f"m{r}.npy")[0]) == world


def _fault_worker(rank, world, port, outdir, mode):
    """Rank 1 misbehaves after step 0: it reports a failure ("raise") or
    stops reporting ("silent"). The other ranks must learn of it through the
    store within the bounded wait and stop before the next step."""
    import datetime
    import json
    from fmha_b200.multi import ShardMonitor
    store = dist.TCPStore("127.0.0.1", port, world, rank == 0,
                          timeout=datetime.timedelta(seconds=20))
    mon = ShardMonitor(store, rank, world, prefix=f"t-{mode}")
    # Start-up handshake: process spawn and imports can skew ranks by seconds,
    # which is not the fault under test.
    mon.report(-1, ok=True)
    assert mon.wait_step(-1, timeout_s=60.0) == ({}, [])
    log = []
    for step in range(3):
        if rank == 1 and step == 1:
            if mode == "raise":
                try:
                    raise RuntimeError("injected shard failure")
                except RuntimeError as e:
                    mon.report(step, ok=False, reason=str(e))
            log.append(("stopped", step))
            break  # leaves between steps, nothing in flight
        mon.report(step, ok=True)
        failed, missing = mon.wait_step(step, timeout_s=1.0)
        log.append((step, sorted(failed), missing))
        if failed or missing:
            break
    with open(os.path.join(outdir, f"f{mode}{rank}.json"), "w") as f:
        json.dump(log, f)
    if rank == 0:
        import time
        time.sleep(0.5)  # keep the store up while the others read


@pytest.mark.parametrize("mode", ["raise", "silent"])
def test_shard_failure_is_detected_on_the_host(tmp_path, mode):
    import json
    world = 3
    mp.spawn(_fault_worker, args=(world, _free_port(), str(tmp_path), mode), nprocs=world,
             join=True)
    for r in (0, 2):
        log = json.load(open(tmp_path / f"f{mode}{r}.json"))
        assert log[0] == [0, [], []]
        step, failed, missing = log[1]
        assert step == 1
        if mode == "raise":
            assert failed == [1] and missing == []
        else:
            assert failed == [] and missing == [1]
        assert len(log) == 2  # stopped before step 2
    assert json.load(open(tmp_path / f"f{mode}1.json"))[-1] == ["stopped", 1]
