"""Lockstep, teacher-forced comparison of engine runners (test infrastructure).

Several runners see the same batches from one scheduler; the leader's
sampled tokens are fed back to all of them, so every runner decodes the same
contexts. At each sampling step this records, per follower and sampled row,
the largest logit difference from the leader (delta) and every token that
differs from the leader's.

A follower's token may differ from the leader's only at a near tie of the
sampler's scores s(v) = logit(v) / T + g(v), where g is the Gumbel noise of
the reference's SplitMix64 stream (kernels/kernels.cu:371-377, 413-431),
identical in both runners. With leader token r and follower token m, the
leader's margin s_L(r) - s_L(m) is at most
  ((l_L(r) - l_F(r)) + (l_F(m) - l_L(m))) / T  <=  2 * delta / T
whenever both samplers return the exact argmax of their own scores (for
T = 0, the same without the division and noise). `explained` records
whether each mismatch satisfies that bound.
"""
from __future__ import annotations

import ctypes

import numpy as np
import torch

M64 = np.uint64(0xFFFFFFFFFFFFFFFF)


def _splitmix64(v):
    with np.errstate(over="ignore"):
        v = (v + np.uint64(0x9E3779B97F4A7C15)) & M64
        v = ((v ^ (v >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)) & M64
        v = ((v ^ (v >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)) & M64
        return v ^ (v >> np.uint64(31))


def gumbel(seed, tokens):
    """g(v) = -log(-log(u)) for the given token ids (float64 of the float32 u)."""
    tokens = np.asarray(tokens, dtype=np.uint64)
    with np.errstate(over="ignore"):
        x = _splitmix64(np.uint64(seed) ^ ((tokens * np.uint64(0xD2B74407B1CE6E93)) & M64))
    u = ((x >> np.uint64(41)).astype(np.float32) + np.float32(0.5)) * np.float32(1.0 / 8388608.0)
    return -np.log(-np.log(u.astype(np.float64)))


def to_c_batch(host, batch):
    """An NvbhBatch over contiguous copies of a Python Batch's arrays."""
    keep = [np.ascontiguousarray(a) for a in (batch.token_ids, batch.positions, batch.sequence_ids,
                                              batch.slot_mapping, batch.block_tables, batch.last_token_indices,
                                              batch.temperatures, np.asarray(batch.seeds, dtype=np.uint64))]
    ptr = [a.ctypes.data if a.size else None for a in keep]
    b = host.NvbhBatch(ptr[0], ptr[1], ptr[2], ptr[3], len(batch.token_ids), ptr[4], len(batch.block_tables),
                       batch.table_stride, ptr[5], ptr[6], ptr[7], len(batch.last_token_indices),
                       int(batch.is_decode))
    return b, keep


class OursRunner:
    """This library's model as a Python-called runner (nvbe_model_run)."""

    def __init__(self, pkg, model):
        self.pkg, self.model = pkg, model

    def run(self, batch):
        b, _keep = to_c_batch(self.pkg.host, batch)
        n = len(batch.last_token_indices)
        out = (ctypes.c_uint32 * max(n, 1))()
        rc = self.pkg.model.library().nvbe_model_run(self.model.c_handle(), ctypes.byref(b), out)
        if rc:
            raise RuntimeError(self.model.last_error())
        return list(out)[:n]

    def last_logits(self):
        return self.model.last_logits()


class Lockstep:
    """Runs `leader` and `followers` (name -> runner) on every batch and
    returns the leader's tokens; see the module docstring."""

    def __init__(self, leader, followers):
        self.leader, self.followers = leader, followers
        self.steps = 0
        self.delta = {n: [] for n in followers}       # per sampled row: max |logit - leader logit|
        self.mean_err = {n: [] for n in followers}    # per sampled row: mean |logit - leader logit|
        self.mismatches = {n: [] for n in followers}  # (step, row, leader tok, follower tok, margin, bound, explained)
        self.samples = 0

    def run(self, batch):
        lead = self.leader.run(batch)
        k = len(lead)
        if k == 0:
            for f in self.followers.values():
                f.run(batch)
            return lead
        self.steps += 1
        self.samples += k
        l_lead = self.leader.last_logits().double()
        for name, f in self.followers.items():
            toks = f.run(batch)
            l_f = f.last_logits().double()
            diff = (l_f - l_lead).abs()
            for row in range(k):
                d = diff[row].max().item()
                self.delta[name].append(d)
                self.mean_err[name].append(diff[row].mean().item())
                r, m = int(lead[row]), int(toks[row])
                if r == m:
                    continue
                T = float(batch.temperatures[row])
                if T > 0:
                    g = gumbel(int(batch.seeds[row]), [r, m])
                    margin = (l_lead[row, r] - l_lead[row, m]).item() / T + (g[0] - g[1])
                    bound = ((l_lead[row, r] - l_f[row, r]) + (l_f[row, m] - l_lead[row, m])).item() / T
                else:
                    margin = (l_lead[row, r] - l_lead[row, m]).item()
                    bound = ((l_lead[row, r] - l_f[row, r]) + (l_f[row, m] - l_lead[row, m])).item()
                self.mismatches[name].append((self.steps, row, r, m, margin, bound, margin <= bound + 1e-3))
        return lead

    def summary(self):
        out = {"sampling_steps": self.steps, "samples": self.samples}
        for n in self.followers:
            mm = self.mismatches[n]
            out[n] = {"max_logit_delta": max(self.delta[n], default=0.0),
                      "mean_logit_err": float(np.mean(self.mean_err[n])) if self.mean_err[n] else 0.0,
                      "token_mismatches": len(mm), "match_rate": 1.0 - len(mm) / max(1, self.samples),
                      "unexplained": [x for x in mm if not x[6]],
                      "largest_mismatch_margin": max((x[4] for x in mm), default=0.0)}
        return out
