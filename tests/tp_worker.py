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


def run(rank, world, port, cfg, items, seqs, steps, queue):
    try:
        import torch
        import torch.distributed as dist

        from atb_llm_study_b200 import capi
        from test_gpu_engine import EngineConfig

        from datetime import timedelta

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
        capi.check(L.b200_comm_create(world, rank, rank, uid, 64 << 20, ctypes.byref(comm)), "comm_create")
        h = ctypes.create_string_buffer(64)
        capi.check(L.b200_comm_ipc_handle(comm, h), "ipc_handle")
        hs = [None] * world
        dist.all_gather_object(hs, h.raw)
        allh = ctypes.create_string_buffer(b"".join(hs), 64 * world)
        capi.check(L.b200_comm_connect(comm, allh), "comm_connect")

        ec = EngineConfig(None, json.dumps(cfg).encode(), rank, 8, 256, 512, 128, 5, 0.02)
        eng = ctypes.c_void_p()
        capi.check(L.b200_engine_create_tp(ctypes.byref(ec), comm, ctypes.byref(eng)), "engine_create_tp")
        for name, a in items:
            a = np.ascontiguousarray(a, np.float32)
            capi.check(L.b200_engine_set_weight(eng, name.encode(), a.ctypes.data, 2, a.size), name)

        V = cfg["vocab_size"]
        Vl = V // world
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
