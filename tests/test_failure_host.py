"""CPU: failure detection of the tensor-parallel group, made on the host (no GPU fault).

* The communicator's bounded settle (non-blocking NCCL, ``ncclCommGetAsyncError`` polled until
  the call settles, ``ncclCommAbort`` after the group's timeout or on an asynchronous error)
  is driven with scripted NCCL results through the library's host-only test hook.
* A rank that exits between steps is noticed by the others on the host, through the
  ``torch.distributed`` store, before their next step is enqueued (world size 2 over gloo).
"""
import ctypes
import json
import os
import socket
import time

import pytest
import torch.multiprocessing as mp

SUCCESS, IN_PROGRESS, REMOTE_ERROR = 0, 7, 6  # ncclSuccess, ncclInProgress, ncclRemoteError


def settle(mpc, states, timeout_ms):
    arr = (ctypes.c_int * len(states))(*states)
    aborted, polls = ctypes.c_int(-1), ctypes.c_int(-1)
    status = mpc.lib().mg_comm_settle_selftest(arr, len(states), timeout_ms, ctypes.byref(aborted),
                                               ctypes.byref(polls))
    return status, aborted.value, polls.value


def test_a_settled_call_is_not_aborted(mpc):
    status, aborted, polls = settle(mpc, [IN_PROGRESS, IN_PROGRESS, SUCCESS], 10_000)
    assert (status, aborted, polls) == (0, 0, 3)


def test_an_asynchronous_error_aborts_the_communicator(mpc):
    status, aborted, polls = settle(mpc, [IN_PROGRESS, REMOTE_ERROR], 10_000)
    assert status == 7 and aborted == 1 and polls == 2  # MG_DRIVER_FAILED
    assert b"aborted" in mpc.lib().mg_last_error()


def test_a_call_that_never_settles_times_out_and_aborts(mpc):
    t0 = time.monotonic()
    status, aborted, polls = settle(mpc, [IN_PROGRESS], 60)
    elapsed = time.monotonic() - t0
    assert status == 8 and aborted == 1 and polls > 1  # MG_DEVICE_UNAVAILABLE
    assert 0.05 <= elapsed < 5.0
    assert b"did not answer within 60 ms" in mpc.lib().mg_last_error()


def test_settle_arguments_are_checked(mpc):
    assert mpc.lib().mg_comm_settle_selftest(None, 0, 10, None, None) == 12
    assert mpc.lib().mg_comm_check(None) == 12
    assert mpc.lib().mg_comm_abort(None) == 12
    assert mpc.lib().mg_comm_wait(None, 10) == 12
    assert mpc.lib().mg_comm_is_aborted(None) == 0


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, leave_after, result_path):
    import sys
    import importlib
    from datetime import timedelta
    import torch.distributed as dist
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, root)
    tp = importlib.import_module("magnetar-provider-cuda_b200.tensor_parallel")
    store = dist.TCPStore("127.0.0.1", port, world, rank == 0, timeout=timedelta(seconds=30))
    mon = tp.StepMonitor(store, rank, world, timeout_s=1.0)
    outcome = {"rank": rank, "steps": [], "lost": None}
    for step in range(4):
        if rank == 1 and step == leave_after:
            break  # leaves between steps, with nothing of its own in flight
        try:
            mon.step(step)
        except tp.PeerLost as e:
            outcome["lost"] = (e.step, e.missing)
            break
        outcome["steps"].append(step)
    if rank == 0:
        with open(result_path, "w") as f:
            json.dump(outcome, f)
        time.sleep(0.2)


def test_a_rank_that_leaves_between_steps_is_noticed_on_the_host(tmp_path):
    path = str(tmp_path / "r.json")
    mp.start_processes(_rank, args=(2, _free_port(), 2, path), nprocs=2, join=True, start_method="spawn")
    with open(path) as f:
        outcome = json.load(f)
    assert outcome["steps"] == [0, 1]
    assert outcome["lost"] == [2, [1]]
