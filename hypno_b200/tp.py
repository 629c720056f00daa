"""Tensor-parallel plumbing for the sm_100a backend.

Sharding (done by hc_model_load for rank r of size S, Megatron style):
  q/k/v_proj  rows of heads [r*nh/S, (r+1)*nh/S) and kv heads [r*nkv/S, ...)
  o_proj      columns of those query heads        -> partial sums, all-reduce
  gate/up     rows [r*im/S, (r+1)*im/S)
  down_proj   the same columns                    -> partial sums, all-reduce
  LM head     vocabulary rows [r*V/S, (r+1)*V/S)  -> all-gather of logits
  embedding   replicated

`shard_plan` restates those ranges for host-side checks; `join` shares the
NCCL unique id over an existing torch.distributed group (gloo or nccl) and
initialises the model's communicator.
"""
import ctypes

import numpy as np

from ._lib import call


def shard_plan(cfg, rank, size):
    """Row / column ranges of every projection kept by `rank` (hidden, heads,
    kv_heads, inter, vocab from the model config dict)."""
    H, nh, nkv, im, V = cfg["hidden"], cfg["heads"], cfg["kv_heads"], cfg["inter"], cfg["vocab"]
    if nh % size or nkv % size or im % size or V % size:
        raise ValueError(f"tensor parallel size {size} must divide heads, kv heads, intermediate and vocab")
    hd = H // nh
    q0, qn = rank * (nh // size) * hd, (nh // size) * hd
    k0, kn = rank * (nkv // size) * hd, (nkv // size) * hd
    f0, fn = rank * (im // size), im // size
    v0, vn = rank * (V // size), V // size
    return {
        "q_rows": (q0, q0 + qn), "kv_rows": (k0, k0 + kn), "o_cols": (q0, q0 + qn),
        "ffn_rows": (f0, f0 + fn), "down_cols": (f0, f0 + fn), "vocab_rows": (v0, v0 + vn),
    }


def new_unique_id():
    buf = (ctypes.c_uint8 * 128)()
    call("hc_comm_unique_id", buf)
    return bytes(buf)


def join(model, rank, size, group=None, timeout_s=60.0):
    """Shares rank 0's NCCL unique id over torch.distributed and joins the
    model's tensor-parallel communicator."""
    import torch.distributed as dist
    obj = [new_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(obj, src=0, group=group)
    uid = np.frombuffer(obj[0], dtype=np.uint8).copy()
    call("hc_comm_init", model.handle, uid.ctypes.data, rank, size, float(timeout_s))
    return obj[0]
