"""Compact rollout history on the device (the reference's DeviceRolloutHistory).

A rollout records, before each ply, one 12,000-byte record per env for its
acting seat (``snapshot``); PPO later draws minibatches of (step, env)
indices and gets back exactly the observation, global features, legal ids
and canonical mask that seat saw (``reconstruct``), rebuilt on the device by
the same observation and legal kernels the rollout used.  This replaces
storing the observations themselves: 366 KB per (step, env) become 12 KB.
"""
from __future__ import annotations

import ctypes

import numpy as np
import torch

from . import _native as N
from .batch import DeviceBatch
from .env import MASK_BYTES, MAX_LEGAL, OBS_CHANNELS, OBS_GLOBAL, _stream_ptr, ensure_device


class RolloutHistory:
    """(num_steps, num_envs) records in one device buffer."""

    def __init__(self, num_steps: int, num_envs: int, device: int = 0):
        if num_steps <= 0 or num_envs <= 0:
            raise ValueError("num_steps and num_envs must be positive")
        ensure_device(device)
        self.device = torch.device("cuda", device)
        self.num_steps, self.num_envs = int(num_steps), int(num_envs)
        self.record_bytes = int(N.lib().jq_history_record_bytes())
        self.buf = torch.empty(self.num_steps * self.num_envs * self.record_bytes, dtype=torch.uint8,
                               device=self.device)
        self.history_bytes = self.buf.numel()
        self._cap = 0
        self._scratch = None

    @property
    def num_records(self) -> int:
        return self.num_steps * self.num_envs

    def snapshot(self, batch: DeviceBatch, step: int, seats: torch.Tensor | None = None) -> None:
        """Record every env of `batch` (observer `seats`, default each env's turn) as `step`."""
        if batch.n != self.num_envs:
            raise ValueError(f"batch has {batch.n} envs, history {self.num_envs}")
        s = None if seats is None else seats.to(device=self.device, dtype=torch.int8).contiguous()
        N.check(N.lib().jq_history_snapshot(ctypes.byref(batch.struct), None if s is None else s.data_ptr(),
                                            self.buf.data_ptr(), int(step), self.num_steps, _stream_ptr()),
                "jq_history_snapshot")

    def _ensure_scratch(self, b: int) -> None:
        if b <= self._cap:
            return
        self._cap = max(b, 2 * self._cap)
        dev = self.device
        self._scratch = DeviceBatch(self._cap, dev)
        self.observers = torch.zeros(self._cap, dtype=torch.int8, device=dev)
        self.counts = torch.zeros(self._cap, dtype=torch.int32, device=dev)
        self.ids = torch.zeros((self._cap, MAX_LEGAL), dtype=torch.int32, device=dev)
        self.mask = torch.zeros((self._cap, MASK_BYTES), dtype=torch.uint8, device=dev)
        self.spatial = torch.empty((self._cap, OBS_CHANNELS, 17, 17), dtype=torch.float32, device=dev)
        self.global_ = torch.empty((self._cap, OBS_GLOBAL), dtype=torch.float32, device=dev)

    def reconstruct(self, flat_indices, show_mode: int = 2) -> dict[str, torch.Tensor]:
        """Rebuild records step * num_envs + env: spatial (B, 317, 17, 17), global (B, 28),
        mask (B, 16641) uint8, counts (B,), ids (B, 512), observers (B,).  The returned
        tensors are views of reusable buffers, overwritten by the next call."""
        idx = torch.as_tensor(np.asarray(flat_indices, dtype=np.int64) if not torch.is_tensor(flat_indices)
                              else flat_indices, dtype=torch.int64).to(self.device).contiguous()
        b = int(idx.numel())
        if b == 0:
            raise ValueError("empty minibatch")
        self._ensure_scratch(b)
        view = self._scratch.view(0, b)
        L, st = N.lib(), _stream_ptr()
        N.check(L.jq_history_restore(self.buf.data_ptr(), self.num_records, idx.data_ptr(), ctypes.byref(view),
                                     self.observers.data_ptr(), st), "jq_history_restore")
        N.check(L.jq_legal(ctypes.byref(view), self.observers.data_ptr(), self.counts.data_ptr(), self.ids.data_ptr(),
                           MAX_LEGAL, self.mask.data_ptr(), st), "jq_legal")
        N.check(L.jq_observe(ctypes.byref(view), self.observers.data_ptr(), 1, int(show_mode), self.spatial.data_ptr(),
                             self.global_.data_ptr(), st), "jq_observe")
        return {"spatial": self.spatial[:b], "global": self.global_[:b], "mask": self.mask[:b],
                "counts": self.counts[:b], "ids": self.ids[:b], "observers": self.observers[:b]}
