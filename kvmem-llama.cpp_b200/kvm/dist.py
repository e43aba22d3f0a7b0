"""Multi-GPU plumbing for libkvm sessions over torch.distributed.

Two ways to spread the reselection path over GPUs, one process per GPU:

* independent sessions (agent sessions): every rank owns whole sessions; there
  is no collective on the data path -- only the timing barrier.  Weak scaling.
* layer split (one large session): rank r owns attention layers
  [l0_r, l1_r).  It scores only its layers (kvm_score_terms), the per-layer
  score terms meet in ONE collective, every rank then holds the same block
  scores, runs the same deterministic top-k and diff, and stages in only its
  own layers' K/V.

The collective comes in two forms:
  "allgather" (default): all-gather the [layers, blocks] f64 terms, then sum
      them in global layer order on each rank -- bit-identical to one GPU
      (the reference sums layers in ascending order,
      src/adapter/llama-memory-kvmem.cpp:2881-2912).
  "allreduce": each rank sums its own layers, then an NCCL all-reduce (sum,
      f64) of the [blocks] vector -- 64 KiB at 8192 blocks; the association of
      the layer sum changes, so scores agree to ~1e-16 relative rather than
      bit for bit.
This module only moves tensors; the device kernels live in libkvm.
"""
from __future__ import annotations

from dataclasses import dataclass


def layer_range(n_layers: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous layer range of `rank`; the first n_layers % world ranks get one more."""
    base, extra = divmod(n_layers, world)
    l0 = rank * base + min(rank, extra)
    return l0, l0 + base + (1 if rank < extra else 0)


@dataclass
class LayerSplit:
    n_layers: int
    rank: int
    world: int
    mode: str = "allgather"
    group: object = None

    def __post_init__(self):
        if self.mode not in ("allgather", "allreduce"):
            raise ValueError(f"unknown combine mode {self.mode!r}")
        self.l0, self.l1 = layer_range(self.n_layers, self.rank, self.world)
        self.counts = [b - a for a, b in (layer_range(self.n_layers, r, self.world)
                                          for r in range(self.world))]

    @property
    def n_local(self) -> int:
        return self.l1 - self.l0

    def _buffers(self, B, dtype, device):
        """Persistent send [rows, B] and receive [world * rows, B] buffers of the
        all-gather (rows = the largest layer share; padding rows stay zero)."""
        import torch
        key = (B, dtype, str(device))
        if getattr(self, "_buf_key", None) != key:
            rows = max(self.counts)
            self._send = torch.zeros((rows, B), dtype=dtype, device=device)
            self._recv = torch.empty((self.world * rows, B), dtype=dtype, device=device)
            self._buf_key = key
        return self._send, self._recv

    def send_buffer(self, B, dtype, device):
        """[n_local, B] view of the all-gather's send buffer: scoring straight
        into it saves the copy in gather_terms."""
        return self._buffers(B, dtype, device)[0][:self.n_local]

    def gather_terms(self, local_terms):
        """[n_local, B] f64 (any device) -> [n_layers, B] in global layer order.
        One all_gather_into_tensor into a persistent buffer; when every rank has
        the same number of layers that buffer already is [n_layers, B] in
        global order."""
        if self.world == 1:
            return local_terms.contiguous()
        import torch
        import torch.distributed as dist
        B = local_terms.shape[1]
        send, recv = self._buffers(B, local_terms.dtype, local_terms.device)
        if local_terms.data_ptr() != send.data_ptr():
            send[:self.n_local].copy_(local_terms)
        dist.all_gather_into_tensor(recv, send, group=self.group)
        rows = send.shape[0]
        if all(c == rows for c in self.counts):
            return recv
        return torch.cat([recv[r * rows:r * rows + c] for r, c in enumerate(self.counts)], dim=0)

    def reduce_partial(self, partial):
        """In-place sum over ranks of each rank's [B] f64 partial layer sum."""
        if self.world == 1:
            return partial
        import torch.distributed as dist
        dist.all_reduce(partial, op=dist.ReduceOp.SUM, group=self.group)
        return partial


def layer_split_scores(sess, split: LayerSplit, terms_local, acc, n_active: int, stream=None):
    """One layer-split scoring round on a libkvm session that holds this rank's
    layers.  terms_local: device f64 [n_local, ldt]; acc: device f64 [>= blocks];
    n_active: layers with a query across all ranks.  Leaves the combined scores
    installed in the session, ready for kvm_select."""
    n_blocks = sess.block_count
    ldt = terms_local.shape[1]
    if split.mode == "allgather" and split.world > 1:
        # score straight into the all-gather's send buffer (ldt = n_blocks)
        send = split.send_buffer(n_blocks, terms_local.dtype, terms_local.device)
        sess.score_terms(0, split.n_local, send.data_ptr(), n_blocks, stream=stream)
        full = split.gather_terms(send)
        sess.reduce_terms(full.data_ptr(), split.n_layers, n_blocks, acc.data_ptr(), stream=stream)
    elif split.mode == "allgather":
        sess.score_terms(0, split.n_local, terms_local.data_ptr(), ldt, stream=stream)
        sess.reduce_terms(terms_local.data_ptr(), split.n_layers, ldt, acc.data_ptr(), stream=stream)
    else:
        sess.score_terms(0, split.n_local, terms_local.data_ptr(), ldt, stream=stream)
        sess.reduce_terms(terms_local.data_ptr(), split.n_local, ldt, acc.data_ptr(), stream=stream)
        split.reduce_partial(acc[:n_blocks])
    sess.set_scores_from_sum(acc.data_ptr(), n_active, stream=stream)
