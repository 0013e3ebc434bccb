"""Cold-store search split by token range over ranks (one process per GPU).

The reference searches one CPU FAISS IndexFlatIP per layer (controller.py:250-293). Here a
layer's cold index can be scanned by `world` ranks at once: rank r scores the entries of its
token range [r*n/world, (r+1)*n/world) of the cold ring (hc_cold_topk, the same arithmetic
as the single-device scan), keeps its best k as (score, global id), and one all-gather of
world*k pairs over NCCL lets every rank merge them (hc_shard_merge) into the exact global
top k (ties to the lower id, i.e. the older entry), because the global top k is a subset of
the union of the ranges' top k. Every rank then splices the same hits (hc_splice_hits).

Decode state and payload are the same on every rank (each rank runs the sequence's decode
on its own copy, so the pooled query needs no broadcast); only the scan is divided. A token
range is a range of ages (0 = the oldest live entry): on a ring that has wrapped it is at most
two runs of contiguous slots (age_runs), searched separately and merged before the exchange.
"""

from __future__ import annotations

import torch

from . import _lib
from ._lib import call, ptr, size


def token_range(n: int, rank: int, world: int) -> tuple[int, int]:
    """Entries [lo, hi) of a cold index of n entries that `rank` of `world` scans."""
    return rank * n // world, (rank + 1) * n // world


def age_runs(head: int, ccap: int, lo: int, hi: int) -> list[tuple[int, int, int]]:
    """Ages [lo, hi) of a cold ring (age 0 = the oldest live entry, at physical slot `head` of
    a ring of ccap slots) as runs of contiguous slots: [(first slot, length, first age)], one
    run, or two when the range crosses the end of the ring, or none when it is empty."""
    if hi <= lo:
        return []
    s0 = (head + lo) % ccap
    n = hi - lo
    first = min(n, ccap - s0)
    runs = [(s0, first, lo)]
    if first < n:
        runs.append((0, n - first, lo + first))
    return runs


def local_topk(index_rows: torch.Tensor, id_base: int, qvec: torch.Tensor, k: int, ws=None, out=None):
    """Exact inner-product top k of index_rows (n, F) fp32 against qvec (F,) fp32, ids
    id_base + row (hc_cold_topk). Returns (scores (k,) fp32, ids (k,) int32) on the device,
    written into `out` = (scores, ids) when given (contiguous views)."""
    dev = qvec.device
    n, F = (int(index_rows.shape[0]), int(index_rows.shape[1])) if index_rows.numel() else (0, int(qvec.numel()))
    if n and (index_rows.stride(1) != 1 or index_rows.stride(0) != F):
        index_rows = index_rows.contiguous()
    nbytes = size("hc_cold_topk_scratch_bytes", n, k)
    scratch = ws.get(nbytes) if ws is not None else torch.empty(nbytes, dtype=torch.uint8, device=dev)
    sc, ids = out if out is not None else (torch.empty(k, dtype=torch.float32, device=dev),
                                           torch.empty(k, dtype=torch.int32, device=dev))
    call("hc_cold_topk", ptr(index_rows) if n else None, n, F, int(id_base), ptr(qvec.contiguous()), int(k), ptr(sc),
         ptr(ids), ptr(scratch), scratch.numel(), _lib.stream_of(dev))
    return sc, ids


def merge_candidates(cand_scores: torch.Tensor, cand_ids: torch.Tensor, n_shards: int, k: int, out_id=None,
                     out_sc=None):
    """Global top k of n_shards lists of k (score, id) candidates (hc_shard_merge); the ids
    and scores go to `out_id` / `out_sc` (contiguous (k,) views) when given."""
    dev = cand_scores.device
    if out_id is None:
        out_id = torch.empty(k, dtype=torch.int32, device=dev)
    if out_sc is None:
        out_sc = torch.empty(k, dtype=torch.float32, device=dev)
    call("hc_shard_merge", ptr(cand_scores.contiguous()), ptr(cand_ids.contiguous()), int(n_shards), int(k),
         ptr(out_id), ptr(out_sc), _lib.stream_of(dev))
    return out_sc, out_id


class ShardedColdSearch:
    """The exchange of a token-range-sharded cold search over a process group.

    search(runs, n, qvecs, k) takes, for each of B sequences, this rank's part of the cold
    index (the ages token_range(n[b], rank, world)) as a list of (rows, first age) runs of
    contiguous index rows (shard.age_runs: one run, or two on a ring that has wrapped) and its
    query vector, and returns the (B, k) global top-k ids (ages) on every rank. Two runs are
    merged on this rank first. One all-gather per search, whatever B (scores and ids travel
    together in one int32 buffer).
    `local` and `merge` default to the CUDA kernels; a test may pass host functions with the
    same contracts to check the exchange without a GPU.
    """

    def __init__(self, group=None, rank: int | None = None, world: int | None = None, local=None, merge=None):
        import torch.distributed as dist
        self.dist = dist if dist.is_available() and dist.is_initialized() else None
        self.group = group
        self.rank = rank if rank is not None else (dist.get_rank(group) if self.dist else 0)
        self.world = world if world is not None else (dist.get_world_size(group) if self.dist else 1)
        self.local = local or local_topk
        self.merge = merge or merge_candidates
        self.ws = None

    def check_k(self, k: int) -> None:
        """The per-rank top k and the merge have limits (hc_cold_topk: k <= 256; hc_shard_merge:
        world * k <= 4096): refuse a lookahead beyond them before any decode runs."""
        if not 1 <= k <= 256:
            raise ValueError(f"sharded cold search needs 1 <= lookahead_k <= 256 (got {k})")
        if self.world * k > 4096:
            raise ValueError(f"sharded cold search needs world * lookahead_k <= 4096 (got {self.world} x {k})")

    def _local_runs(self, runs, qvec, k, out):
        """This rank's top k over its runs of index rows into out = (scores, ids) views."""
        cuda = self.local is local_topk
        if not runs:
            runs = [(qvec.new_zeros((0, qvec.numel())), 0)]
        if len(runs) == 1:
            rows, base = runs[0]
            if cuda:
                local_topk(rows, base, qvec, k, self.ws, out=out)
            else:
                s, i = self.local(rows, base, qvec, k)
                out[0].copy_(s)
                out[1].copy_(i)
            return
        cs = torch.empty((len(runs), k), dtype=torch.float32, device=qvec.device)
        ci = torch.empty((len(runs), k), dtype=torch.int32, device=qvec.device)
        for j, (rows, base) in enumerate(runs):
            if cuda:
                local_topk(rows, base, qvec, k, self.ws, out=(cs[j], ci[j]))
            else:
                s, i = self.local(rows, base, qvec, k)
                cs[j], ci[j] = s, i
        if self.merge is merge_candidates:
            merge_candidates(cs.view(-1), ci.view(-1), len(runs), k, out_id=out[1], out_sc=out[0])
        else:
            s, i = self.merge(cs.view(-1), ci.view(-1), len(runs), k)
            out[0].copy_(s)
            out[1].copy_(i)

    def search(self, runs, n, qvecs, k: int) -> torch.Tensor:
        self.check_k(k)
        B = len(runs)
        dev = qvecs.device
        # one buffer of (scores | ids) per sequence, so that a single all-gather exchanges both
        packed = torch.empty((B, 2 * k), dtype=torch.int32, device=dev)
        sc, ids = packed.view(torch.float32)[:, :k], packed[:, k:]
        for b in range(B):
            self._local_runs(runs[b], qvecs[b], k, (sc[b], ids[b]))
        if self.world == 1:
            return ids.contiguous()  # one range: its top k (sorted, ties to the lower id) is the answer
        allp = torch.empty((self.world * B, 2 * k), dtype=torch.int32, device=dev)
        self.dist.all_gather_into_tensor(allp, packed, group=self.group)
        allp = allp.view(self.world, B, 2 * k)
        all_sc, all_id = allp.view(torch.float32)[:, :, :k], allp[:, :, k:]
        out = torch.empty((B, k), dtype=torch.int32, device=dev)
        for b in range(B):
            if self.merge is merge_candidates:
                merge_candidates(all_sc[:, b].reshape(-1), all_id[:, b].reshape(-1), self.world, k, out_id=out[b])
            else:
                _, out[b] = self.merge(all_sc[:, b].reshape(-1), all_id[:, b].reshape(-1), self.world, k)
        return out
