"""Rank body of the tensor-parallel tests (imported by spawned processes).

Each rank bootstraps a b200_comm_t over a gloo process group (NCCL unique id
and CUDA IPC handles exchanged as objects), builds the tensor-parallel engine
from whole weights, runs a packed prefill and a few greedy decode steps, and
returns its logits shards and tokens to the parent through a queue."""

import ctypes
import json
import os
import sys
import traceback

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))
sys.path.insert(0, HERE)


def _bootstrap(rank, world, port, sym_bytes):
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    from atb_llm_study_b200 import capi

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=120))
    torch.cuda.set_device(rank)
    L = capi.lib()
    uid = ctypes.create_string_buffer(128)
    if rank == 0:
        capi.check(L.b200_comm_unique_id(uid), "unique_id")
    box = [uid.raw]
    dist.broadcast_object_list(box, src=0)
    uid = ctypes.create_string_buffer(box[0], 128)
    comm = ctypes.c_void_p()
    capi.check(L.b200_comm_create(world, rank, rank, uid, sym_bytes, ctypes.byref(comm)), "comm_create")
    h = ctypes.create_string_buffer(64)
    capi.check(L.b200_comm_ipc_handle(comm, h), "ipc_handle")
    hs = [None] * world
    dist.all_gather_object(hs, h.raw)
    allh = ctypes.create_string_buffer(b"".join(hs), 64 * world)
    capi.check(L.b200_comm_connect(comm, allh), "comm_connect")
    return L, capi, dist, comm


def run(rank, world, port, cfg, items, seqs, steps, mode, queue, limits=None):
    try:
        import torch

        from test_gpu_engine import EngineConfig

        L, capi, dist, comm = _bootstrap(rank, world, port, 64 << 20)
        ec = EngineConfig(None, json.dumps(cfg).encode(), rank, *(limits or (8, 256, 512)), 128, 5, 0.02)
        eng = ctypes.c_void_p()
        create = L.b200_engine_create_ep if mode == "ep" else L.b200_engine_create_tp
        capi.check(create(ctypes.byref(ec), comm, ctypes.byref(eng)), "engine_create_" + mode)
        for name, a in items:
            a = np.ascontiguousarray(a, np.float32)
            capi.check(L.b200_engine_set_weight(eng, name.encode(), a.ctypes.data, 2, a.size), name)

        V = cfg["vocab_size"]
        Vl = V if mode == "ep" else V // world
        if mode == "ep":
            seqs = seqs[rank]
        n = len(seqs)
        ids = np.concatenate(seqs).astype(np.int64)
        lens = np.array([len(s) for s in seqs], np.int32)
        slots = np.arange(n, dtype=np.int32)
        nxt = np.zeros(n, np.int64)
        lg = torch.empty(n, Vl, dtype=torch.bfloat16, device=f"cuda:{rank}")
        capi.check(L.b200_engine_prefill(eng, ids.ctypes.data, 0, lens.ctypes.data, slots.ctypes.data, n, None,
                                         nxt.ctypes.data, 0, lg.data_ptr()), "prefill")
        torch.cuda.synchronize()
        out = {"prefill": (lg.float().cpu().numpy(), nxt.copy()), "decode": []}
        for step in range(steps):
            o = np.zeros(n, np.int64)
            lgd = torch.empty(n, Vl, dtype=torch.bfloat16, device=f"cuda:{rank}")
            capi.check(L.b200_engine_decode(eng, nxt.ctypes.data, 0, slots.ctypes.data, n, o.ctypes.data, 0,
                                            lgd.data_ptr()), f"decode {step}")
            torch.cuda.synchronize()
            out["decode"].append((lgd.float().cpu().numpy(), nxt.copy(), o.copy()))
            nxt = o
        bits = ctypes.c_uint(0)
        capi.check(L.b200_device_error_read(ctypes.addressof(bits), 1, None), "error_read")
        out["errors"] = bits.value
        dist.barrier()
        L.b200_engine_destroy(eng)
        L.b200_comm_destroy(comm)
        dist.destroy_process_group()
        queue.put((rank, out))
    except Exception:
        queue.put((rank, traceback.format_exc()))


def ep_kernels(rank, world, port, E, k, H, T, skip_expert, queue):
    """Route this rank's T random tokens to k distinct experts (never
    `skip_expert`), group them with b200_moe_permute into the symmetric send
    area, dispatch into the symmetric result area (identity experts: the
    received rows are the results), combine with a residual, and return
    everything the parent checks."""
    try:
        import torch

        L, capi, dist, comm = _bootstrap(rank, world, port, 16 << 20)
        dev = f"cuda:{rank}"
        rng = np.random.default_rng(50 + rank)
        choices = [e for e in range(E) if e != skip_expert]
        ids = np.stack([rng.choice(choices, k, replace=False) for _ in range(T)]).astype(np.int32)
        w = rng.random((T, k)).astype(np.float32)
        x = torch.from_numpy(rng.standard_normal((T, H)).astype(np.float32)).to(torch.bfloat16).to(dev)
        res = torch.from_numpy(rng.standard_normal((T, H)).astype(np.float32)).to(torch.bfloat16).to(dev)
        b0, b1, bb = ctypes.c_void_p(), ctypes.c_void_p(), ctypes.c_int64()
        capi.check(L.b200_comm_info(comm, None, None, ctypes.byref(b0), ctypes.byref(b1), ctypes.byref(bb)), "info")
        send_off = b0.value
        send_rows = b0.value + (64 << 10)
        send_cap = T * k
        recv_cap = world * 64 * k  # every rank routes at most 64 tokens here
        idd = torch.from_numpy(ids).to(dev)
        wd = torch.from_numpy(w).to(dev)
        pos = torch.empty(T * k, dtype=torch.int32, device=dev)
        src = torch.empty(T * k, dtype=torch.int32, device=dev)
        wsb = L.b200_moe_permute_workspace_bytes(T, k, E)
        ws = torch.empty(max(wsb, 4), dtype=torch.uint8, device=dev)
        st = torch.cuda.current_stream().cuda_stream
        capi.check(L.b200_moe_permute(idd.data_ptr(), T, k, E, x.data_ptr(), H, H, send_rows, send_off,
                                      pos.data_ptr(), src.data_ptr(), ws.data_ptr(), wsb, st), "permute")
        recv_off = torch.empty(E // world + 1, dtype=torch.int32, device=dev)
        row_base = torch.empty(E, dtype=torch.int32, device=dev)
        capi.check(L.b200_ep_dispatch(comm, send_off, send_rows, send_cap, E, H, b1.value, recv_cap,
                                      recv_off.data_ptr(), row_base.data_ptr(), st), "dispatch")
        out = torch.empty(T, H, dtype=torch.bfloat16, device=dev)
        capi.check(L.b200_ep_combine(comm, b1.value, recv_cap, row_base.data_ptr(), send_off, idd.data_ptr(),
                                     wd.data_ptr(), pos.data_ptr(), T, k, E, H, res.data_ptr(), None, out.data_ptr(),
                                     None, None, 1e-6, st), "combine")
        torch.cuda.synchronize()
        ro = recv_off.cpu().numpy()
        nrecv = int(ro[-1])
        recv = torch.empty(max(nrecv, 1), H, dtype=torch.bfloat16, device=dev)
        if nrecv:  # the received rows, read back from the symmetric result area
            from cuda.bindings import runtime as rt

            err, = rt.cudaMemcpy(recv.data_ptr(), b1.value, nrecv * H * 2, rt.cudaMemcpyKind.cudaMemcpyDeviceToDevice)
            assert err == rt.cudaError_t.cudaSuccess, err
        recv = recv[:nrecv]
        bits = ctypes.c_uint(0)
        capi.check(L.b200_device_error_read(ctypes.addressof(bits), 1, None), "error_read")
        result = dict(ids=ids, w=w, x=x.float().cpu().numpy(), res=res.float().cpu().numpy(),
                      out=out.float().cpu().numpy(), recv=recv.float().cpu().numpy(), recv_off=ro,
                      row_base=row_base.cpu().numpy(), errors=bits.value)
        dist.barrier()
        L.b200_comm_destroy(comm)
        dist.destroy_process_group()
        queue.put((rank, result))
    except Exception:
        queue.put((rank, traceback.format_exc()))


def wait_timeout(rank, world, port, queue):
    """Rank 0 enters the fused all-reduce; rank 1 never does (it waits on the
    host).  Rank 0's bounded flag wait must give up after ~2 s, set the
    device error word's timeout bit and return, leaving its context usable;
    then both ranks tear down."""
    try:
        import time

        import torch

        L, capi, dist, comm = _bootstrap(rank, world, port, 16 << 20)
        dev = f"cuda:{rank}"
        out = {"errors": 0}
        if rank == 0:
            H, T = 512, 4
            hidden = torch.ones(T, H, dtype=torch.bfloat16, device=dev)
            bits = ctypes.c_uint(0)
            capi.check(L.b200_device_error_read(ctypes.addressof(bits), 1, None), "error_read")  # clear
            t0 = time.time()
            capi.check(L.b200_comm_allreduce_rmsnorm(comm, 0, T, H, hidden.data_ptr(), None, None, 1e-6,
                                                     torch.cuda.current_stream().cuda_stream), "allreduce_rmsnorm")
            torch.cuda.synchronize()
            out["seconds"] = time.time() - t0
            capi.check(L.b200_device_error_read(ctypes.addressof(bits), 1, None), "error_read")
            out["timeout_bits"] = bits.value
            # the context still runs work
            x = torch.randn(8, 64, device=dev).to(torch.bfloat16)
            w = torch.ones(64, dtype=torch.bfloat16, device=dev)
            y = torch.empty_like(x)
            capi.check(L.b200_rmsnorm(x.data_ptr(), None, w.data_ptr(), y.data_ptr(), None, 8, 64, 64, 1e-6,
                                      torch.cuda.current_stream().cuda_stream), "rmsnorm")
            torch.cuda.synchronize()
            ref = (x.float() * torch.rsqrt(x.float().pow(2).mean(-1, keepdim=True) + 1e-6)).to(torch.bfloat16)
            out["context_ok"] = bool(torch.allclose(y.float(), ref.float(), atol=2e-2, rtol=2e-2))
        dist.barrier()  # rank 1 waits here, on the host, while rank 0's kernel times out
        L.b200_comm_destroy(comm)
        dist.destroy_process_group()
        queue.put((rank, out))
    except Exception:
        queue.put((rank, traceback.format_exc()))
