# SPDX-License-Identifier: MIT
"""A CPU model of the vocabulary-shard stages (test infrastructure).

EmuEngine stands in for beamgrad_b200.vocab_sharding.CudaEngine so that the host side of
the vocabulary-sharded decode -- the stage order, the collectives between the stages, the
stalled-row rescans -- runs on gloo ranks without a GPU. Each stage keeps the device
stages' contract on the exchange buffers (row maxima, packed rows, resume / stalled,
rescanned lists); the per-step selection itself is the oracle's single step
(oracle.oracle_step) over rows holding only the candidates the merged records (or the
rescans) provide, so a decode matches the oracle's full decode only when the records and
the rescans are enough -- which is what the test checks. float32 inputs, no n-gram
blocking or repetition penalty.
"""

from __future__ import annotations

import ctypes as C

import numpy as np
import torch

from beamgrad_b200 import _abi as A
from beamgrad_b200 import vocab_sharding as vs
from oracle import oracle


def make_key(x: float, index: int) -> int:
    """The engine's 64-bit key: order-preserving bits of x (+0 for -0), then ~index."""
    u = int(np.array([np.float32(x) + np.float32(0.0)], np.float32).view(np.uint32)[0])
    ordered = (~u & 0xFFFFFFFF) if u & 0x80000000 else (u | 0x80000000)
    return (ordered << 32) | (0xFFFFFFFF - index)


def key_x(key: int) -> np.float32:
    o = key >> 32
    u = (o & 0x7FFFFFFF) if o & 0x80000000 else (~o & 0xFFFFFFFF)
    return np.array([u], np.uint32).view(np.float32)[0]


def key_index(key: int) -> int:
    return 0xFFFFFFFF - (key & 0xFFFFFFFF)


class EmuEngine:
    def __init__(self):
        self.lib = A.load()  # the plan is host-only and needs no device
        self.olib = oracle.oracle_lib()

    def plan(self, args, from_logits, world, rank, shard_list_len):
        p = A.VocabShardPlan()
        A.check(self.lib.dbs_cuda_vshard_plan(C.byref(args), int(from_logits), world, rank, shard_list_len,
                                              C.byref(p)), "vshard plan")
        return p

    def run(self, stage: str, d) -> None:
        getattr(self, stage)(d)

    # ------------------------------------------------------------------ helpers
    @staticmethod
    def _meta(d):
        s = d.settings
        steps = d.steps.numpy() if d.steps is not None else np.full(d.B, d.T, np.int32)
        eos = s["eos_token"]
        eos_set = set(([eos] + list(s["extra_eos"])) if eos >= 0 else [])
        return steps, eos, eos_set, s["min_length"]

    @staticmethod
    def _read_rows(d, steps):
        for b in range(d.B):
            for t in range(d.T):
                for k in range(d.K):
                    if t < steps[b] and (t > 0 or k == 0):
                        yield b, t, k, (b * d.T + t) * d.K + k

    # ------------------------------------------------------------------ stages
    def scan(self, d):
        assert d.shard.dtype == torch.float32 and d.settings["no_repeat_ngram_size"] == 0
        assert d.settings["repetition_penalty"] <= 1.0
        steps, eos, eos_set, min_len = self._meta(d)
        p = d.plan
        LS, RW = p.shard_list_len, p.row_words
        key_off = RW - LS
        x = d.shard.numpy()
        toks = vs.shard_tokens(d.V, d.world, d.rank).numpy()
        banned = d.banned.numpy().astype(bool) if d.banned is not None else np.zeros(d.V, bool)
        ex = np.zeros((d.B * d.T * d.K, RW), np.uint64)
        rmax = np.full(d.B * d.T * d.K, -np.inf, np.float32)
        rmin = np.full(d.B * d.T * d.K, np.inf, np.float32)
        for b, t, k, rowi in self._read_rows(d, steps):
            row = x[b, t, k]
            if row.size == 0:
                continue
            with np.errstate(invalid="ignore"):
                below = row < np.inf
            invalid = bool((~below).any())
            rmax[rowi] = row[below].max() if below.any() else -np.inf
            rmin[rowi] = np.fmin.reduce(row)
            mask_eos = eos >= 0 and t + 1 < min_len
            elig = below & (row > -np.inf) & ~banned[toks]
            if mask_eos:
                elig &= ~np.isin(toks, list(eos_set))
            idx = np.nonzero(elig)[0]
            order = sorted(idx, key=lambda i: (-float(row[i]), int(toks[i])))[:LS]
            cnt = len(order)
            ex[rowi, 0] = int(invalid) | (2 if cnt >= LS else 0) | (cnt << 8)
            for j, i in enumerate(order):
                ex[rowi, key_off + j] = make_key(row[i], int(toks[i]))
        d.row_max.copy_(torch.from_numpy(rmax))
        d.row_min.copy_(torch.from_numpy(rmin))
        d.exchange.copy_(torch.from_numpy(ex.view(np.int64)))
        d.resume.zero_()
        d.stalled.zero_()
        d.out["invalid"].zero_()
        raw = np.full((d.B, d.K), -np.inf, np.float32)
        raw[:, 0] = 0.0
        d.emu = {"raw": raw, "len": np.zeros((d.B, d.K), np.int32), "fin": np.zeros((d.B, d.K), np.uint8),
                 "final": {}}

    def lanes(self, d):
        steps, _, _, _ = self._meta(d)
        L = d.plan.lanes
        x = d.shard.numpy()
        ex = d.exchange.numpy().view(np.uint64)
        mx_all = d.row_max.numpy()
        for b, t, k, rowi in self._read_rows(d, steps):
            out = np.zeros(L, np.float32)
            row = np.ascontiguousarray(x[b, t, k])
            self.olib.oracle_shard_lanes(row.ctypes.data_as(C.c_void_p), row.size, d.world, float(mx_all[rowi]),
                                         out.ctypes.data_as(C.c_void_p))
            ex[rowi, 1:1 + L // 2] = out.view(np.uint64)

    def merge(self, d):
        steps, _, _, _ = self._meta(d)
        p = d.plan
        rows, RW, LS, LIST, L = d.B * d.T * d.K, p.row_words, p.shard_list_len, p.list_len, p.lanes
        key_off = RW - LS
        allx = d.exchange_all.numpy().view(np.uint64).reshape(d.world, rows, RW)
        mx_all = d.row_max.numpy()
        d.emu["rec"], d.emu["lse"] = {}, {}
        for b, t, k, rowi in self._read_rows(d, steps):
            lse = 0.0
            if d.from_logits:
                lanes = np.concatenate([allx[r, rowi, 1:1 + L // 2].view(np.float32) for r in range(d.world)])
                lse = self.olib.oracle_lse_from_lanes(np.ascontiguousarray(lanes).ctypes.data_as(C.c_void_p),
                                                      float(mx_all[rowi]))
            infos = [int(allx[r, rowi, 0]) for r in range(d.world)]
            lists = [[int(v) for v in allx[r, rowi, key_off:key_off + (infos[r] >> 8)]] for r in range(d.world)]
            full = [bool(i & 2) for i in infos]
            bound = max([lst[-1] for lst, f in zip(lists, full) if f and lst], default=0)
            keys = sorted((v for lst in lists for v in lst if v >= bound), reverse=True)[:LIST]
            info = int(any(i & 1 for i in infos)) | (2 if any(full) else 0) | (len(keys) << 8)
            d.emu["rec"][rowi] = (keys, info)
            d.emu["lse"][rowi] = np.float32(lse)

    def select(self, d):
        steps, eos, eos_set, min_len = self._meta(d)
        p, s = d.plan, d.settings
        LIST = p.list_len
        resume = d.resume.numpy()
        stalled = d.stalled.numpy().view(np.uint32)
        n_rescan = int(d.call.buffers.n_rescan)
        slots = d.rescan_slot.numpy() if n_rescan else None
        rescan_all = d.rescan_all.numpy().view(np.uint64).reshape(d.world, n_rescan, d.K) if n_rescan else None
        e = d.emu
        for b in range(d.B):
            t0 = int(resume[b])
            for t in range(t0, d.T):
                active = t < steps[b]
                lp_rows = np.full((d.K, d.V), -np.inf, np.float32)
                stall = []
                d.out["row_lse"][b, t] = 0.0
                for k in range(d.K):
                    rowi = (b * d.T + t) * d.K + k
                    pr = e["raw"][b, k]
                    read = active and (t > 0 or k == 0) and np.isfinite(pr) and not (eos >= 0 and e["fin"][b, k])
                    if not read:
                        continue
                    keys, info = e["rec"][rowi]
                    lse = e["lse"][rowi]
                    if info & 1:
                        d.out["invalid"][b] = 1
                    d.out["row_lse"][b, t, k] = float(lse) if d.from_logits else 0.0
                    cnt = info >> 8
                    partial = cnt >= LIST or bool(info & 2)
                    xs = [key_x(v) for v in keys]
                    lps = [np.float32(x - lse) if d.from_logits else x for x in xs]
                    raws = [np.float32(pr + lp) if np.isfinite(lp) else -np.inf for lp in lps]
                    raw_last = raws[-1] if (partial and cnt > 0) else -np.inf
                    above = sum(1 for r in raws if r > raw_last)
                    exact = e["len"][b, k] == t and (not partial or above >= d.K)
                    if exact:
                        for v, lp in zip(keys, lps):
                            lp_rows[k, key_index(v)] = lp
                    else:
                        stall.append(k)
                if stall:
                    if t == t0 and slots is not None and all(slots[b * d.K + k] >= 0 for k in stall):
                        for k in stall:
                            rowi = (b * d.T + t) * d.K + k
                            lse = e["lse"][rowi]
                            for r in range(d.world):
                                for v in rescan_all[r, slots[b * d.K + k]]:
                                    v = int(v)
                                    if v:
                                        x = key_x(v)
                                        lp_rows[k, key_index(v)] = np.float32(x - lse) if d.from_logits else x
                    else:
                        resume[b] = t
                        stalled[b] = 0
                        for k in stall:
                            stalled[b, k // 32] |= np.uint32(1 << (k % 32))
                        break
                self._emit(d, b, t, active, lp_rows, eos, min_len, s)
            else:
                resume[b] = d.T

    def _emit(self, d, b, t, active, lp_rows, eos, min_len, s):
        e = d.emu
        o = d.out
        if active:
            pb = oracle.Problem(np.ascontiguousarray(lp_rows[None, None]), eos=eos, min_length=min_len,
                                alpha=s["length_penalty_alpha"], extra_eos=list(s["extra_eos"]))
            step = oracle.oracle_step(pb, e["raw"][b:b + 1], e["len"][b:b + 1], e["fin"][b:b + 1], None)
            for name in ("tokens", "parents", "lengths", "scores", "raw_scores", "from_logprob"):
                o[name][b, t] = torch.from_numpy(np.ascontiguousarray(step[name][0, 0]))
            e["raw"][b], e["len"][b], e["fin"][b] = step["state_raw"][0], step["state_lengths"][0], \
                step["state_finished"][0]
            e["final"][b] = (step["final_scores"][0], step["final_raw_scores"][0], step["final_lengths"][0])
        else:
            o["tokens"][b, t] = -1
            o["parents"][b, t] = -1
            o["lengths"][b, t] = 0
            o["scores"][b, t] = -np.inf
            o["raw_scores"][b, t] = -np.inf
            o["from_logprob"][b, t] = 0
        if t == d.T - 1:
            fs, fr, fl = e["final"][b]
            o["final_scores"][b] = torch.from_numpy(fs.copy())
            o["final_raw_scores"][b] = torch.from_numpy(fr.copy())
            o["final_lengths"][b] = torch.from_numpy(fl.copy())

    def rescan(self, d):
        steps, eos, eos_set, min_len = self._meta(d)
        x = d.shard.numpy()
        toks = vs.shard_tokens(d.V, d.world, d.rank).numpy()
        banned = d.banned.numpy().astype(bool) if d.banned is not None else np.zeros(d.V, bool)
        out = np.zeros((int(d.call.buffers.n_rescan), d.K), np.uint64)
        resume = d.resume.numpy()
        for slot, bk in enumerate(d.rescan_rows.numpy()):
            b, k = divmod(int(bk), d.K)
            t = int(resume[b])
            rowi = (b * d.T + t) * d.K + k
            pr = d.emu["raw"][b, k]
            lse = d.emu["lse"][rowi]
            mask_eos = eos >= 0 and d.emu["len"][b, k] + 1 < min_len
            row = x[b, t, k]
            cands = []
            for i, v in enumerate(toks):
                xv = row[i]
                if not (xv < np.inf) or xv == -np.inf or banned[v] or (mask_eos and v in eos_set):
                    continue
                lp = np.float32(xv - lse) if d.from_logits else xv
                raw = np.float32(pr + lp)
                if raw != -np.inf:
                    cands.append((make_key(raw, k * d.V + int(v)), make_key(xv, int(v))))
            cands.sort(reverse=True)
            for j, (_, xk) in enumerate(cands[:d.K]):
                out[slot, j] = xk
        d.rescan.copy_(torch.from_numpy(out.view(np.int64)))
