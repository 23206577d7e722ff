"""Benchmark of the B200 paged-KV data path.

Headline: batch-decode PagedAttention KV GB/s on the Llama-3-70B head shape
(config 5: 64 Q / 8 KV heads, head_size 128, bf16 KV, FP32 Q/O, batch 256,
sequence lengths uniform in [4096, 32768], block 16, randomly fragmented
pools). With N GPUs the KV heads are sharded: rank g owns KV heads
[g*8/N, (g+1)*8/N) and their Q heads, with its own pool and block tables; the
timed region has no collective. `value` = KV bytes of all ranks / max-over-
ranks time per step (strong scaling: the job is fixed, N splits it).

The same JSON line carries: `e2e` (the same metric through the drop-in C++
API, paged_attention_batch_host with Q and O in pinned host memory, H2D + D2H
inside the timed region), `roofline` of the decode kernel, `cpu_baseline`
(the reference's CPU path on a bounded sample, rank 0 at N=1, with the
reference's own GPU kernels timed beside this build's), clocks, and
`secondary` lines: config 5 as a serving decode step (append + fused write
and decode through BatchDecodeSession), KV-write tokens/s and gather GB/s on
config 2 (64 sequences x 8192 tokens, 256 new tokens per step, odd/even
fragmented 65,536-page pool), decode GB/s on config 3 (Llama-3-8B heads,
batch 64, lengths in [512, 8192]), config 2's shapes over 32 layers (layer-
batched write and gather) and config 4's prefix-sharing prefill (8 x 4096
tokens in one batched tcgen05 launch; rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]

Inputs are synthetic (seeded). Decode, gather and prefill inputs are far
larger than the 126 MB L2, so no flush is needed between timed steps; the
write launches rotate over slot/input sets that together exceed L2, and are
reported per launch and over graph-captured back-to-back launches.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "decode paged-attn KV GB/s (% HBM peak) + KV-write tokens/s at 1/2/4/8 B200"
HBM_FALLBACK_GBS = 6650.0
DATASHEET_GBS = 7700.0


def load_peak():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
    return HBM_FALLBACK_GBS, "fallback"


def load_bf16_peak():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return float(json.loads(p.read_text())["bf16_tflops"]), "measured"
    return 1590.0, "fallback"


def traffic_ratio(kernel: str):
    """DRAM bytes per algorithmic byte from a committed ncu summary, if any."""
    p = ROOT / "profiles" / "ncu_traffic.json"
    if not p.exists():
        return None, None
    d = json.loads(p.read_text()).get(kernel)
    if not d:
        return None, None
    return float(d["dram_bytes_per_algorithmic_byte"]), d.get("capture")


# ------------------------------------------------------------------ ranks ---

class Ranks:
    def __init__(self, gpus: int):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        if self.world > 1 and self.world != gpus:
            raise SystemExit(f"--gpus {gpus} but WORLD_SIZE={self.world}")
        self.dist = None

    @classmethod
    def this_rank_only(cls) -> "Ranks":
        """A one-rank view (no collectives) for work one rank does alone."""
        r = cls.__new__(cls)
        r.world, r.rank, r.local, r.dist = 1, 0, int(os.environ.get("LOCAL_RANK", "0")), None
        return r

    def init_gpu(self):
        import datetime

        import torch

        torch.cuda.set_device(self.local)
        if self.world > 1:
            import torch.distributed as dist

            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=900),
                                    device_id=torch.device("cuda", self.local))
            self.dist = dist

    def barrier(self):
        if self.dist is not None:
            self.dist.barrier()

    def reduce(self, x: float, op: str) -> float:
        if self.dist is None:
            return x
        import torch

        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX if op == "max" else self.dist.ReduceOp.SUM)
        return float(t.item())

    def close(self):
        if self.dist is not None:
            self.dist.barrier()
            self.dist.destroy_process_group()


# ----------------------------------------------------------------- clocks ---

class Clocks:
    """Samples nvidia-smi clocks and throttle reasons during a region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    NAMES = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

    def __init__(self, device: int):
        self.device, self.proc, self.path = device, None, None

    def __enter__(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.device}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "50"],
                                         stdout=fd, stderr=subprocess.DEVNULL)
            os.close(fd)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        sm, mx, reasons = [], [], set()
        for line in Path(self.path).read_text().splitlines():
            r = [x.strip() for x in line.split(",")]
            try:
                sm.append(float(r[1]))
                mx.append(float(r[2]))
            except (ValueError, IndexError):
                continue
            for name, val in zip(self.NAMES, r[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------- raw memory ---

_RT = None


def cudart():
    global _RT
    if _RT is None:
        import torch

        torch.cuda.init()
        _RT = ctypes.CDLL("libcudart.so.12")
        _RT.cudaMemcpy.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int]
    return _RT


def d2h(addr: int, out: np.ndarray) -> None:
    assert cudart().cudaMemcpy(out.ctypes.data, addr, out.nbytes, 2) == 0


# ------------------------------------------------------------ workloads ---

def fill_cache(kv, storage, seqs, seed: int, chunk_tokens: int = 1 << 16):
    """Writes N(0,1) bf16 K/V into every reserved slot through kvfx_write."""
    import torch

    desc = kv.cache_descriptor(storage)
    lay = storage.layout()
    heads, hd, bs = lay.num_kv_heads(), lay.head_size(), lay.block_size()
    gen = torch.Generator(device="cuda")
    gen.manual_seed(seed)
    parts = []
    for s in seqs:
        n = s.num_tokens()
        tbl = np.array(kv.build_read_block_table(s), np.uint64)
        t = np.arange(n, dtype=np.uint64)
        parts.append(tbl[t // bs] * bs + t % bs)
    slots = np.concatenate(parts)
    kbuf = torch.empty(chunk_tokens * heads * hd, dtype=torch.bfloat16, device="cuda")
    vbuf = torch.empty_like(kbuf)
    for start in range(0, len(slots), chunk_tokens):
        part = slots[start:start + chunk_tokens]
        n = len(part)
        kbuf[: n * heads * hd].normal_(generator=gen)
        vbuf[: n * heads * hd].normal_(generator=gen)
        sd = torch.from_numpy(part.view(np.int64)).cuda()
        kv.check(kv.lib.kvfx_write(ctypes.byref(desc), kbuf.data_ptr(), vbuf.data_ptr(), sd.data_ptr(), n, None),
                 "fill kvfx_write")
    torch.cuda.synchronize()


class Decode:
    """One rank's shard of a batch-decode config."""

    def __init__(self, kv, w, cfg: dict, rank: int, world: int):
        import torch

        self.kv, self.cfg = kv, cfg
        assert cfg["kv_heads"] % world == 0
        self.kvh = cfg["kv_heads"] // world
        self.qh = cfg["q_heads"] // world
        self.hd, self.bs = cfg["head_size"], cfg["block_size"]
        self.lens = w.config_lengths(cfg).astype(np.uint64)
        self.batch = len(self.lens)
        pages = int(sum((int(l) + self.bs - 1) // self.bs for l in self.lens))
        cap = cfg.get("pool_pages") or (1 << int(math.ceil(math.log2(pages * 1.25))))
        self.b = w.decode_batch_on_pool(cap, self.bs, self.lens, seed=cfg["seed"] * 131 + rank, mode="random")
        dev = torch.cuda.current_device()
        self.storage = kv.PagedKVStorage(self.b.pool, self.kvh, self.hd, kv.DType.BFloat16, dev)
        fill_cache(kv, self.storage, self.b.sequences, seed=cfg["seed"] * 7 + rank)
        self.table_np, self.width = self.b.table()
        self.table = torch.from_numpy(self.table_np.view(np.int64)).cuda()
        self.lens_d = torch.from_numpy(self.lens.view(np.int64)).cuda()
        gen = torch.Generator(device="cuda")
        gen.manual_seed(cfg["seed"] * 3 + rank)
        self.q = torch.randn(self.batch * self.qh * self.hd, generator=gen, device="cuda", dtype=torch.float32)
        self.o = torch.empty_like(self.q)
        self.desc = kv.cache_descriptor(self.storage)
        self.max_len = int(self.lens.max())
        self.pps = cfg.get("pages_per_split") or kv.lib.kvfx_decode_pages_per_split(
            ctypes.byref(self.desc), self.batch, self.qh, self.max_len, int(self.lens.sum()))
        ws = kv.lib.kvfx_decode_workspace_bytes(ctypes.byref(self.desc), self.batch, self.qh, self.max_len, self.pps)
        self.ws = torch.zeros(max(int(ws), 16), dtype=torch.uint8, device="cuda")
        self.kv_bytes = int(self.lens.sum()) * self.kvh * self.hd * 2 * 2
        self.alg_bytes = self.kv_bytes + 2 * self.q.numel() * 4 + self.batch * (self.width + 1) * 8

    def launch(self, stream: int | None) -> None:
        rc = self.kv.lib.kvfx_decode(ctypes.byref(self.desc), self.q.data_ptr(), self.o.data_ptr(),
                                     self.table.data_ptr(), self.lens_d.data_ptr(), self.batch, self.width, self.qh,
                                     self.max_len, self.pps, self.ws.data_ptr(), self.ws.numel(), stream)
        self.kv.check(rc, "kvfx_decode")

    def host_sample(self, requests):
        """Pages of `requests` copied to a compact host cache (for the CPU leg)."""
        page_bytes = self.storage.layout().page_bytes()
        ids = [self.table_np[r, :(int(self.lens[r]) + self.bs - 1) // self.bs] for r in requests]
        uniq = np.unique(np.concatenate(ids))
        remap = {int(p): i for i, p in enumerate(uniq)}
        hk = np.empty((len(uniq), page_bytes), np.uint8)
        hv = np.empty_like(hk)
        for i, p in enumerate(uniq):
            d2h(self.storage.key_base() + int(p) * page_bytes, hk[i])
            d2h(self.storage.value_base() + int(p) * page_bytes, hv[i])
        width = max(len(x) for x in ids)
        table = np.zeros((len(requests), width), np.uint64)
        for j, x in enumerate(ids):
            table[j, :len(x)] = [remap[int(p)] for p in x]
        q = self.q.view(self.batch, -1)[list(requests)].cpu().numpy().reshape(-1)
        o = self.o.view(self.batch, -1)[list(requests)].cpu().numpy().reshape(-1)
        return hk.reshape(-1), hv.reshape(-1), len(uniq), table, self.lens[list(requests)].copy(), q, o


def time_launches(launch, steps: int, warmup: int, ranks: Ranks):
    """Device time of each of `steps` launches (CUDA events on the launching
    stream), after `warmup` untimed ones; barrier + synchronize on both sides."""
    import torch

    stream = torch.cuda.Stream()
    sp = stream.cuda_stream
    with torch.cuda.stream(stream):
        for _ in range(warmup):
            launch(sp)
    torch.cuda.synchronize()
    ranks.barrier()
    torch.cuda.synchronize()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(steps + 1)]
    with torch.cuda.stream(stream):
        ev[0].record(stream)
        for i in range(steps):
            launch(sp)
            ev[i + 1].record(stream)
    torch.cuda.synchronize()
    ranks.barrier()
    per = [ev[i].elapsed_time(ev[i + 1]) for i in range(steps)]
    return per, ev[0].elapsed_time(ev[steps])


def e2e_decode(kv, wl: Decode, steps: int, warmup: int):
    """Same metric end to end from host buffers. Headline: one
    paged_attention_batch_host call per step (Q from pinned host memory,
    uploaded per row chunk ahead of that chunk's kernel; the lengths uploaded
    and the device-resident page table refreshed by the call - unchanged rows
    re-send nothing; O written into pinned host memory by the kernels;
    synchronous). Beside it: the device-buffer API with an
    explicit Q copy before and O copy after (the reference's call shape)."""
    import torch

    q_host = wl.q.cpu().pin_memory()
    o_host = torch.empty_like(q_host).pin_memory()
    seqs = wl.b.sequences

    def step_host():
        kv.paged_attention_batch_host(wl.storage, seqs, q_host, o_host, wl.qh)

    def step_device():
        wl.q.copy_(q_host, non_blocking=True)
        kv.paged_attention_batch(wl.storage, seqs, wl.q, wl.o, wl.qh)
        o_host.copy_(wl.o, non_blocking=True)
        torch.cuda.current_stream().synchronize()

    def timed(step):
        for _ in range(warmup):
            step()
        torch.cuda.synchronize()
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        wall = time.perf_counter()
        t0.record()
        for _ in range(steps):
            step()
        t1.record()
        torch.cuda.synchronize()
        wall = time.perf_counter() - wall
        return max(t0.elapsed_time(t1), wall * 1e3) / steps

    ms_device = timed(step_device)
    ms = timed(step_host)
    # What each call uploads besides Q: the lengths and the page-table entries
    # that changed since the previous call (the table stays on the device).
    table_bytes = kv.paged_attention_batch_table_upload_bytes(wl.storage)
    return ms, q_host.numel() * 4 + table_bytes, o_host.numel() * 4, ms_device


def decode_step(kv, wl: Decode, steps: int, warmup: int, ranks: Ranks) -> dict:
    """Config 5 as a serving decode step: every sequence appends one token.

    e2e: BatchDecodeSession.step_host (host page bookkeeping with
    copy-on-write, 16 bytes per row of lengths and slots uploaded, the step's
    new K/V rows and Q uploaded from pinned host memory per row chunk, fused
    write + decode launches over the device-resident block table writing O
    into pinned host memory), all inside the timed region; beside it, step()
    on device buffers with explicit copies before and after. Device: the fused launch alone, repeated on the state
    after the last step (it rewrites the same rows), next to a plain decode
    launch over the same table and lengths."""
    import torch

    seqs = wl.b.sequences
    # The pool holds exactly the prefilled pages; hand back enough held pages
    # for the steps' new pages (at most one per sequence per step).
    spare = min(len(wl.b.holders), 2 * wl.batch)
    for h in wl.b.holders[:spare]:
        wl.b.pool.free(h)
    del wl.b.holders[:spare]
    n = wl.batch * wl.kvh * wl.hd
    gen = torch.Generator(device="cuda")
    gen.manual_seed(wl.cfg["seed"] * 11 + ranks.rank)
    k_dev = torch.randn(n, generator=gen, device="cuda").to(torch.bfloat16)
    v_dev = torch.randn(n, generator=gen, device="cuda").to(torch.bfloat16)
    k_host, v_host = k_dev.cpu().pin_memory(), v_dev.cpu().pin_memory()
    q_host = wl.q.cpu().pin_memory()
    o_host = torch.empty_like(q_host).pin_memory()
    sess = kv.BatchDecodeSession(wl.storage, seqs, wl.qh)

    def step_device():
        k_dev.copy_(k_host, non_blocking=True)
        v_dev.copy_(v_host, non_blocking=True)
        wl.q.copy_(q_host, non_blocking=True)
        sess.step(k_dev, v_dev, wl.q, wl.o)
        o_host.copy_(wl.o, non_blocking=True)
        torch.cuda.current_stream().synchronize()

    def step_host():
        sess.step_host(k_host, v_host, q_host, o_host)

    def timed(step):
        for _ in range(warmup):
            step()
        torch.cuda.synchronize()
        ranks.barrier()
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        wall = time.perf_counter()
        t0.record()
        for _ in range(steps):
            step()
        t1.record()
        torch.cuda.synchronize()
        wall = time.perf_counter() - wall
        ranks.barrier()
        return max(t0.elapsed_time(t1), wall * 1e3) / steps

    dev_api_ms = timed(step_device)
    e2e_ms = timed(step_host)

    lens = np.array([s.num_tokens() for s in seqs], np.uint64)
    slots = np.array(kv.build_slot_mapping([(s, s.num_tokens() - 1) for s in seqs]), np.uint64)
    lens_d = torch.from_numpy(lens.view(np.int64)).cuda()
    slots_d = torch.from_numpy(slots.view(np.int64)).cuda()
    width, table = sess.table_width(), sess.device_table()
    max_len = int(lens.max())
    pps = kv.lib.kvfx_decode_pages_per_split(ctypes.byref(wl.desc), wl.batch, wl.qh, max_len, int(lens.sum()))
    ws_bytes = kv.lib.kvfx_decode_workspace_bytes(ctypes.byref(wl.desc), wl.batch, wl.qh, max_len, pps)
    ws = torch.zeros(max(int(ws_bytes), 16), dtype=torch.uint8, device="cuda")

    def fused(stream):
        kv.check(kv.lib.kvfx_decode_append(ctypes.byref(wl.desc), k_dev.data_ptr(), v_dev.data_ptr(),
                                           slots_d.data_ptr(), wl.q.data_ptr(), wl.o.data_ptr(), table,
                                           lens_d.data_ptr(), wl.batch, width, wl.qh, max_len, pps, ws.data_ptr(),
                                           ws.numel(), stream), "kvfx_decode_append")

    def plain(stream):
        kv.check(kv.lib.kvfx_decode(ctypes.byref(wl.desc), wl.q.data_ptr(), wl.o.data_ptr(), table,
                                    lens_d.data_ptr(), wl.batch, width, wl.qh, max_len, pps, ws.data_ptr(),
                                    ws.numel(), stream), "kvfx_decode")

    _, tot_f = time_launches(fused, steps, warmup, ranks)
    _, tot_p = time_launches(plain, steps, warmup, ranks)
    if kv.device_status(torch.cuda.current_device()) != 0:
        raise RuntimeError("decode step: a kernel flagged an out-of-range id or a timed-out wait")
    fused_ms = ranks.reduce(tot_f / steps, "max")
    plain_ms = ranks.reduce(tot_p / steps, "max")
    e2e_ms = ranks.reduce(e2e_ms, "max")
    dev_api_ms = ranks.reduce(dev_api_ms, "max")
    kv_bytes = ranks.reduce(float(int(lens.sum()) * wl.kvh * wl.hd * 2 * 2), "sum")
    tokens = wl.batch
    world = ranks.world
    return {"workload": "config5 decode step: 256 sequences append one token each (copy-on-write, new pages), "
                        "fused KV write + decode over a device-resident block table",
            "e2e_ms_per_step": e2e_ms, "e2e_tokens_per_s": tokens / (e2e_ms * 1e-3),
            "e2e_kv_gbs": kv_bytes / (e2e_ms * 1e-3) / 1e9,
            "e2e_h2d_bytes_per_step": world * (2 * k_host.numel() * 2 + q_host.numel() * 4 + 2 * tokens * 8),
            "e2e_d2h_bytes_per_step": world * o_host.numel() * 4,
            "api": "kvflux::v2::BatchDecodeSession::step_host (pinned host K/V/Q in, O out)",
            "device_api_ms_per_step": dev_api_ms,
            "fused_ms_per_launch": fused_ms, "fused_kv_gbs": kv_bytes / (fused_ms * 1e-3) / 1e9,
            "plain_decode_ms_per_launch": plain_ms, "table_width": width}


class WriteGather:
    """Config 2 on one rank's KV-head shard."""

    def __init__(self, kv, w, cfg: dict, rank: int, world: int):
        import torch

        self.kv = kv
        self.heads = cfg["kv_heads"] // world
        self.hd, self.bs = cfg["head_size"], cfg["block_size"]
        nseq, pre, new = cfg["sequences"], cfg["prefill"], cfg["new_tokens"]
        self.total_len = pre + new
        lens = [self.total_len] * nseq
        b = w.decode_batch_on_pool(cfg["pool_pages"], self.bs, lens, seed=cfg["seed"] + rank, mode="odd")
        self.b = b
        dev = torch.cuda.current_device()
        self.storage = kv.PagedKVStorage(b.pool, self.heads, self.hd, kv.DType.BFloat16, dev)
        fill_cache(kv, self.storage, b.sequences, seed=cfg["seed"] * 5 + rank)
        self.desc = kv.cache_descriptor(self.storage)
        # The step's 256 slots: the last `new` positions of every sequence.
        self.slots_np = np.array(kv.build_slot_mapping([(s, p) for s in b.sequences
                                                        for p in range(pre, pre + new)]), np.uint64)
        self.n = len(self.slots_np)
        self.slots = torch.from_numpy(self.slots_np.view(np.int64)).cuda()
        step_bytes = self.n * self.heads * self.hd * 2 * 2 * 2 + self.n * 8
        # Timed write launches rotate over `rot` slot sets (the step's slots,
        # then each sequence's `new` positions before them, ...) with their own
        # input rows, so that one rotation touches more than the 126 MB L2.
        self.rot = int(min(pre // new, max(2, -(-2 * 126_000_000 // step_bytes))))
        self.rot_slots = [self.slots] + [
            torch.from_numpy(np.array(kv.build_slot_mapping([(s, p) for s in b.sequences
                                                             for p in range(pre - new * r, pre - new * r + new)]),
                                      np.uint64).view(np.int64)).cuda() for r in range(1, self.rot)]
        gen = torch.Generator(device="cuda")
        gen.manual_seed(cfg["seed"] + 17 * rank)
        rows = self.n * self.heads * self.hd
        self.k_rot = torch.randn(self.rot * rows, generator=gen, device="cuda").to(torch.bfloat16)
        self.v_rot = torch.randn_like(self.k_rot, dtype=torch.float32).to(torch.bfloat16)
        self.k_new, self.v_new = self.k_rot[:rows], self.v_rot[:rows]
        self.turn = 0
        table, self.width = b.table()
        self.table = torch.from_numpy(table.view(np.int64)).cuda()
        self.lens = torch.full((nseq,), self.total_len, dtype=torch.int64, device="cuda")
        self.nseq = nseq
        per = self.total_len * self.heads * self.hd
        self.k_out = torch.empty(nseq * per, dtype=torch.bfloat16, device="cuda")
        self.v_out = torch.empty_like(self.k_out)
        ptrs_k = np.array([self.k_out.data_ptr() + i * per * 2 for i in range(nseq)], np.uint64)
        ptrs_v = np.array([self.v_out.data_ptr() + i * per * 2 for i in range(nseq)], np.uint64)
        self.pk = torch.from_numpy(ptrs_k.view(np.int64)).cuda()
        self.pv = torch.from_numpy(ptrs_v.view(np.int64)).cuda()
        self.write_bytes = self.n * self.heads * self.hd * 2 * 2 * 2 + self.n * 8  # read+write K,V + slots
        self.gather_bytes = 2 * 2 * nseq * per * 2 + table.nbytes  # read+write K,V + table

    def write(self, stream):
        r = self.turn % self.rot
        self.turn += 1
        off = r * self.n * self.heads * self.hd * 2
        self.kv.check(self.kv.lib.kvfx_write(ctypes.byref(self.desc), self.k_rot.data_ptr() + off,
                                             self.v_rot.data_ptr() + off, self.rot_slots[r].data_ptr(), self.n,
                                             stream), "kvfx_write")

    def gather(self, stream):
        self.kv.check(self.kv.lib.kvfx_gather_batch(ctypes.byref(self.desc), self.table.data_ptr(),
                                                    self.lens.data_ptr(), self.nseq, self.width, self.pk.data_ptr(),
                                                    self.pv.data_ptr(), stream), "kvfx_gather_batch")

    def gather_one_by_one(self, stream, tma: bool):
        """Every sequence gathered by its own call: kvfx_gather (the
        single-sequence entry point read_paged_kv uses: TMA tensor copies) or
        kvfx_gather_batch over that one row (the 16-byte load/store kernel)."""
        per = self.total_len * self.heads * self.hd * 2
        for r in range(self.nseq):
            if tma:
                self.kv.check(self.kv.lib.kvfx_gather(ctypes.byref(self.desc), self.table.data_ptr() + r * self.width * 8,
                                                      self.total_len, self.k_out.data_ptr() + r * per,
                                                      self.v_out.data_ptr() + r * per, stream), "kvfx_gather")
            else:
                self.kv.check(self.kv.lib.kvfx_gather_batch(ctypes.byref(self.desc),
                                                            self.table.data_ptr() + r * self.width * 8,
                                                            self.lens.data_ptr() + r * 8, 1, self.width,
                                                            self.pk.data_ptr() + r * 8, self.pv.data_ptr() + r * 8,
                                                            stream), "kvfx_gather_batch")

    def graph_write_ms(self, launches: int = 100) -> float:
        """Per-launch time of `launches` back-to-back writes captured in a CUDA graph."""
        import torch

        s = torch.cuda.Stream()
        with torch.cuda.stream(s):
            self.write(s.cuda_stream)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            for _ in range(launches):
                self.write(s.cuda_stream)
        for _ in range(3):
            g.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reps = 10
        e0.record()
        for _ in range(reps):
            g.replay()
        e1.record()
        torch.cuda.synchronize()
        del g
        return e0.elapsed_time(e1) / (reps * launches)

    def e2e_write_ms(self, steps: int = 20) -> tuple[float, int]:
        import torch

        kh = self.k_new.cpu().pin_memory()
        vh = self.v_new.cpu().pin_memory()
        slots = [int(x) for x in self.slots_np]

        def step():
            self.k_new.copy_(kh, non_blocking=True)
            self.v_new.copy_(vh, non_blocking=True)
            self.kv.write_paged_kv(self.storage, self.k_new, self.v_new, slots)

        for _ in range(3):
            step()
        torch.cuda.synchronize()
        t = time.perf_counter()
        for _ in range(steps):
            step()
        torch.cuda.synchronize()
        return (time.perf_counter() - t) * 1e3 / steps, 2 * kh.numel() * 2 + len(slots) * 8


def graph_ms(launch, ranks: Ranks, launches: int = 50, reps: int = 5) -> float:
    """Per-launch device time of `launches` back-to-back launches captured in
    one CUDA graph (max over ranks): the device rate without the host's
    per-launch cost, for kernels about as short as a host launch."""
    import torch

    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        launch(s.cuda_stream)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=s):
        for _ in range(launches):
            launch(s.cuda_stream)
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    ranks.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        graph.replay()
    e1.record()
    torch.cuda.synchronize()
    del graph
    return ranks.reduce(e0.elapsed_time(e1) / (reps * launches), "max")


def layer_batches(kv, w, rank: int, world: int, ranks: Ranks, layers: int = 32, steps: int = 50, warmup: int = 5,
                  graph: bool = True, tokens: int = 1024) -> dict:
    """Config 2's step across a model's layers (Llama-3-8B: 32 layers, 8 KV
    heads x 128, bf16), one PagedKVStorage per layer on one odd/even
    fragmented pool of 8192 pages: 64 sequences of 1024 tokens. Write: the
    step's 256 new tokens (the last 4 of each sequence) into every layer in
    one kvfx_write_layers launch. Gather: every sequence's K/V of every layer
    to contiguous per-layer runs in one kvfx_gather_layers launch. The caches
    hold whatever the allocation held: the timing does not depend on the
    values (the tests check the bytes). Successive write launches rotate over
    `rot` slot sets (each sequence's last 4 positions, the 4 before them, ...)
    and as many input buffers, so that one rotation touches more bytes than
    the 126 MB L2 holds and every launch reads and writes HBM. `tokens`
    shortens the sequences (and the pool with them) for profiling runs: the
    write's bytes do not depend on it."""
    import torch

    heads, hd, bs = 8 // world, 128, 16
    nseq, total, new = 64, tokens, 4
    pool_pages = 8192 if tokens == 1024 else 2 * nseq * (-(-tokens // bs)) + 2
    b = w.decode_batch_on_pool(pool_pages, bs, [total] * nseq, seed=0xC0F2 + rank, mode="odd")
    dev = torch.cuda.current_device()
    stores = [kv.PagedKVStorage(b.pool, heads, hd, kv.DType.BFloat16, dev) for _ in range(layers)]
    arr = (kv.KvfxCache * layers)(*[kv.cache_descriptor(st) for st in stores])
    row = heads * hd * 2
    rot = min(total // new, max(2, -(-2 * 126_000_000 // max(1, layers * nseq * new * row * 2 * 2))))
    slot_sets = [np.array(kv.build_slot_mapping([(s, p) for s in b.sequences
                                                 for p in range(total - new * (r + 1), total - new * r)]), np.uint64)
                 for r in range(rot)]
    n = len(slot_sets[0])
    slots_d = [torch.from_numpy(sl.view(np.int64)).cuda() for sl in slot_sets]
    gen = torch.Generator(device="cuda")
    gen.manual_seed(0xC0F2 * 3 + rank)
    k_new = torch.randn(rot * layers * n * heads * hd, generator=gen, device="cuda").to(torch.bfloat16)
    v_new = torch.randn_like(k_new, dtype=torch.float32).to(torch.bfloat16)
    in_bytes = layers * n * row  # one launch's K (or V) input
    table, width = b.table()
    table_d = torch.from_numpy(table.view(np.int64)).cuda()
    lens_d = torch.full((nseq,), total, dtype=torch.int64, device="cuda")
    per_layer = total * row
    k_out = torch.empty(nseq * layers * per_layer, dtype=torch.uint8, device="cuda")
    v_out = torch.empty_like(k_out)
    kp = torch.tensor([k_out.data_ptr() + i * layers * per_layer for i in range(nseq)], dtype=torch.int64,
                      device="cuda")
    vp = torch.tensor([v_out.data_ptr() + i * layers * per_layer for i in range(nseq)], dtype=torch.int64,
                      device="cuda")

    turn = [0]

    def write(stream):
        r = turn[0] % rot
        turn[0] += 1
        kv.check(kv.lib.kvfx_write_layers(arr, layers, k_new.data_ptr() + r * in_bytes, v_new.data_ptr() + r * in_bytes,
                                          n * row, slots_d[r].data_ptr(), n, stream), "kvfx_write_layers")

    def gather(stream):
        kv.check(kv.lib.kvfx_gather_layers(arr, layers, table_d.data_ptr(), lens_d.data_ptr(), nseq, width,
                                           kp.data_ptr(), vp.data_ptr(), per_layer, stream), "kvfx_gather_layers")

    _, tot_w = time_launches(write, steps, warmup, ranks)
    _, tot_g = time_launches(gather, max(1, steps // 5), 3, ranks)
    wg_ms = float("nan")
    if graph:
        wg_ms = graph_ms(write, ranks)
    w_ms = ranks.reduce(tot_w / steps, "max")
    g_ms = ranks.reduce(tot_g / max(1, steps // 5), "max")

    peak = load_peak()[0]
    w_bytes = ranks.reduce(float(layers * (n * row * 2 * 2 + n * 8)), "sum")
    g_bytes = ranks.reduce(float(layers * nseq * total * row * 2 * 2 + table.nbytes), "sum")
    out = {"workload": f"{layers} layers x config2 shapes (8 KV heads x 128 bf16), one storage per layer on one "
                       f"{pool_pages}-page odd/even pool, 64 sequences x {total} tokens",
           "write_tokens": n, "write_rotation": f"{rot} slot/input sets, {rot * w_bytes / world / 1e6:.0f} MB "
                                                 f"touched per rotation (L2 126 MB)",
           "write_ms_per_launch": w_ms, "write_layer_tokens_per_s": layers * n / (w_ms * 1e-3),
           "write_gbs": w_bytes / (w_ms * 1e-3) / 1e9,
           "write_frac_of_peak": w_bytes / (w_ms * 1e-3) / 1e9 / (peak * world),
           "write_graph_ms_per_launch": wg_ms if graph else None,
           "write_graph_gbs": w_bytes / (wg_ms * 1e-3) / 1e9 if graph else None,
           "write_graph_frac_of_peak": w_bytes / (wg_ms * 1e-3) / 1e9 / (peak * world) if graph else None,
           "gather_ms_per_launch": g_ms, "gather_gbs": g_bytes / (g_ms * 1e-3) / 1e9,
           "gather_frac_of_peak": g_bytes / (g_ms * 1e-3) / 1e9 / (peak * world)}
    del stores, k_out, v_out
    return out


def reference_gpu_sample(kv, w, rows: int = 4, reps: int = 3):
    """Part of the baseline leg (rank 0, N = 1, not with --no-cpu).
    The reference's own GPU kernels on this B200 beside this build's, on
    the same sample: config 3's first `rows` requests (Llama-3-8B heads, bf16),
    the same page ids and inputs, both driven through the v2 C++ API
    (write_paged_kv of every token, then paged_attention_batch; synchronous
    calls timed on the host clock: the first write, and medians of `reps`
    repeats of each call). None when the reference
    GPU library is not built."""
    import oracle
    import torch

    if oracle.ref_gpu() is None:
        return None
    cfg = w.CONFIG3
    kvh, qh, hd, bs = cfg["kv_heads"], cfg["q_heads"], cfg["head_size"], cfg["block_size"]
    lens = [int(x) for x in w.config_lengths(cfg)[:rows]]
    nb = sum((l + bs - 1) // bs for l in lens) + 16
    order = w.permutation(cfg["seed"], np.arange(nb))
    total = sum(lens)
    k = w.encode(w.normal(cfg["seed"] + 1, total * kvh * hd), "bfloat16")
    v = w.encode(w.normal(cfg["seed"] + 2, total * kvh * hd), "bfloat16")
    q = w.normal(cfg["seed"] + 3, rows * qh * hd)
    o_ref, ref_write_ms, ref_ms = oracle.ref_gpu_decode(torch.cuda.current_device(), nb, bs, order, kvh, qh, hd, 1,
                                                        lens, k, v, q, reps=reps)
    pool = kv.PhysicalBlockPool(nb, bs)
    w.fragment_pool(pool, order)
    st = kv.PagedKVStorage(pool, kvh, hd, kv.DType.BFloat16, torch.cuda.current_device())
    seqs = []
    for L in lens:
        s_ = kv.SequenceState(len(seqs) + 1, pool)
        s_.append_tokens(L)
        seqs.append(s_)
    slots = kv.build_slot_mapping([(s_, t) for s_ in seqs for t in range(s_.num_tokens())])
    kd, vd = torch.from_numpy(k.view(np.int16)).cuda(), torch.from_numpy(v.view(np.int16)).cuda()
    torch.cuda.synchronize()
    wtimes = []
    for _ in range(reps + 1):  # the first call, then `reps` repeats of the same write
        t = time.perf_counter()
        kv.write_paged_kv(st, kd, vd, slots)
        wtimes.append((time.perf_counter() - t) * 1e3)
    qd = torch.from_numpy(q).cuda()
    o = torch.empty_like(qd)
    times = []
    for _ in range(reps + 2):
        t = time.perf_counter()
        kv.paged_attention_batch(st, seqs, qd, o, qh)
        times.append((time.perf_counter() - t) * 1e3)
    ours_ms = statistics.median(times[2:])
    kv_bytes = total * kvh * hd * 2 * 2
    return {"workload": f"config3 decode, requests 0-{rows - 1} (lengths {lens}), bf16; the reference's CUDA kernels "
                        "(compiled from its sources for sm_100a) and this build's, both through the v2 C++ API",
            "reference_decode_ms": ref_ms, "ours_decode_ms": ours_ms, "decode_speedup": ref_ms / ours_ms,
            "reference_kv_gbs": kv_bytes / (ref_ms * 1e-3) / 1e9, "ours_kv_gbs": kv_bytes / (ours_ms * 1e-3) / 1e9,
            "reference_write_ms": ref_write_ms[1], "ours_write_ms": statistics.median(wtimes[1:]),
            "reference_first_write_ms": ref_write_ms[0], "ours_first_write_ms": wtimes[0],
            "write_timing": "write_paged_kv of every token (one call), host clock around the synchronous call: "
                            "median of repeats of the same call; ours includes the Python binding's slot-list "
                            "conversion",
            "write_tokens": total,
            "max_abs_diff": float(np.abs(o.cpu().numpy() - o_ref).max())}


class Prefill:
    """Config 4 on one GPU: 8 sequences x 4096 tokens, 32 Q / 8 KV heads,
    hd 128, bf16. Sequence 0 is written to 2056 tokens (128 full pages + a
    partial page of 8), forked three times; each fork appends one token with a
    copy-on-write of the shared partial page, then grows to 4096 with its own
    K/V. Sequences 4-7 are independent. One step = the 8 causal prefill
    attentions (query_tokens = kv_tokens = 4096)."""

    def __init__(self, kv, w, cfg: dict):
        import torch

        self.kv = kv
        L, H, G, hd, bs = cfg["tokens"], cfg["kv_heads"], cfg["q_heads"] // cfg["kv_heads"], cfg["head_size"], 16
        self.L, self.qh, self.hd = L, H * G, hd
        pages = cfg["sequences"] * (L // bs + 1) + 16
        self.pool = kv.PhysicalBlockPool(pages, bs)
        dev = torch.cuda.current_device()
        self.storage = kv.PagedKVStorage(self.pool, H, hd, kv.DType.BFloat16, dev)
        gen = torch.Generator(device="cuda")
        gen.manual_seed(cfg["seed"])

        def write(seq, lo, hi):
            n = hi - lo
            k = torch.randn(n * H * hd, generator=gen, device="cuda").to(torch.bfloat16)
            v = torch.randn(n * H * hd, generator=gen, device="cuda").to(torch.bfloat16)
            kv.write_paged_kv(self.storage, k, v, kv.build_slot_mapping([(seq, t) for t in range(lo, hi)]))

        shared = cfg["shared_prefix"]
        base = kv.SequenceState(0, self.pool)
        base.append_tokens(shared)
        write(base, 0, shared)
        self.seqs = [base] + [base.fork_shared(i) for i in range(1, cfg["shared_group"])]
        self.cow_copies = 0
        for s in self.seqs[1:]:
            loc = kv.append_token_cow(self.storage, s)  # byte-exact copy of the shared partial page
            self.cow_copies += int(loc.offset_in_block != 0)
            write(s, shared, shared + 1)
        base.append_tokens(1)
        write(base, shared, shared + 1)
        for s in self.seqs:
            s.append_tokens(L - shared - 1)
            write(s, shared + 1, L)
        for i in range(cfg["shared_group"], cfg["sequences"]):
            s = kv.SequenceState(i, self.pool)
            s.append_tokens(L)
            write(s, 0, L)
            self.seqs.append(s)
        self.tables = [torch.from_numpy(np.array(kv.build_read_block_table(s), np.uint64).view(np.int64)).cuda()
                       for s in self.seqs]
        self.q = torch.randn(L * self.qh * hd, generator=gen, device="cuda")
        self.o = torch.empty_like(self.q)
        self.desc = kv.cache_descriptor(self.storage)
        self.flops = len(self.seqs) * 2.0 * hd * L * (L + 1) * self.qh  # causal QK^T + PV

    def launch(self, stream):
        for t in self.tables:
            rc = self.kv.lib.kvfx_attention(ctypes.byref(self.desc), self.q.data_ptr(), self.o.data_ptr(),
                                            t.data_ptr(), self.L, self.L, self.qh, None, 0, stream)
            self.kv.check(rc, "kvfx_attention")

    def launch_batch(self, stream):
        """The same 8 attentions as one kvfx_attention_batch call (one
        persistent launch; each sequence has its own O buffer)."""
        import torch

        if not hasattr(self, "_batch"):
            n = len(self.tables)
            table = torch.stack(self.tables)
            outs = [torch.empty_like(self.q) for _ in range(n)]
            self._batch = (table, outs, (ctypes.c_void_p * n)(*[self.q.data_ptr()] * n),
                           (ctypes.c_void_p * n)(*[o.data_ptr() for o in outs]), (ctypes.c_uint64 * n)(*[self.L] * n))
        table, _, qp, op, lens = self._batch
        rc = self.kv.lib.kvfx_attention_batch(ctypes.byref(self.desc), len(self.tables), qp, op, table.data_ptr(),
                                              table.shape[1], lens, lens, self.qh, None, 0, stream)
        self.kv.check(rc, "kvfx_attention_batch")


# ----------------------------------------------------------- CPU baseline ---

def cpu_threads() -> int:
    try:
        return max(1, len(os.sched_getaffinity(0)))
    except AttributeError:
        return os.cpu_count() or 1


def cpu_decode_sample(hk, hv, nb, kvh, bs, hd, table, lens, qh, q, budget_s: float = 15.0):
    """Times the reference CPU path (gather + reference_attention per request,
    one std::thread per request slice) on the sample; returns
    (KV GB/s, seconds, kind, threads, requests used, outputs, single-core KV
    GB/s of the one-request calibration run)."""
    import oracle

    threads = cpu_threads()
    use_ref = oracle.ref() is not None
    fn = oracle.ref_decode_batch if use_ref else None

    def run(count):
        t = time.perf_counter()
        if use_ref:
            out = oracle.ref_decode_batch(hk, hv, 1, kvh, bs, hd, table, lens, qh, q, first=0, count=count,
                                          threads=min(threads, count))
        else:
            out = oracle.decode_batch(hk, hv, 1, nb, kvh, bs, hd, table, lens, qh, q, first=0, count=count,
                                      threads=min(threads, count))
        return time.perf_counter() - t, out

    del fn
    # Calibrate on one request, then size the sample to the time budget.
    t1, _ = run(1)
    per_wave = max(t1, 1e-3)
    waves = max(1, int(budget_s / per_wave))
    count = min(len(lens), max(1, waves * threads))
    secs, out = run(count)
    kv_bytes = int(lens[:count].sum()) * kvh * hd * 2 * 2
    one_core = int(lens[0]) * kvh * hd * 2 * 2 / max(t1, 1e-9) / 1e9
    return kv_bytes / secs / 1e9, secs, "reference" if use_ref else "port", min(threads, count), count, out, one_core


# ------------------------------------------------------------- reference ---

def reference_arm(args, ranks: Ranks) -> int:
    """The reference's own CPU implementation of batch decode (its
    reference_attention, compiled from its sources, after the gather its GPU
    kernel does, restated on the CPU) on this box's host cores, on config 5's
    shapes; each step is a bounded sample of requests (one per thread)."""
    if ranks.rank != 0:
        return 0
    import importlib.util

    import oracle

    # The seeded generators by file path: importing the kvflux_b200 package
    # would load this build's native library into the reference's process.
    spec = importlib.util.spec_from_file_location("kvflux_synth", ROOT / "kvflux_b200" / "synth.py")
    w = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(w)

    cfg = w.CONFIG5
    threads = cpu_threads()
    lens_all = w.config_lengths(cfg).astype(np.uint64)
    count = min(len(lens_all), threads)
    lens = lens_all[:count]
    kvh, qh, hd, bs = cfg["kv_heads"], cfg["q_heads"], cfg["head_size"], cfg["block_size"]
    pages = [(int(l) + bs - 1) // bs for l in lens]
    nb = sum(pages)
    ids = w.permutation(cfg["seed"], np.arange(nb))
    width = max(pages)
    table = np.zeros((count, width), np.uint64)
    k = 0
    for r, p in enumerate(pages):
        table[r, :p] = ids[k:k + p]
        k += p
    n = nb * kvh * bs * hd
    hk = w.f32_to_bf16_bits(w.normal(cfg["seed"] + 1, n))
    hv = w.f32_to_bf16_bits(w.normal(cfg["seed"] + 2, n))
    q = w.normal(cfg["seed"] + 3, count * qh * hd)
    kind = "reference" if oracle.ref() is not None else "port"

    def step():
        if kind == "reference":
            oracle.ref_decode_batch(hk, hv, 1, kvh, bs, hd, table, lens, qh, q, threads=threads)
        else:
            oracle.decode_batch(hk, hv, 1, nb, kvh, bs, hd, table, lens, qh, q, threads=threads)

    for _ in range(args.warmup):
        step()
    t = time.perf_counter()
    for _ in range(args.steps):
        step()
    secs = (time.perf_counter() - t) / args.steps
    kv_bytes = int(lens.sum()) * kvh * hd * 2 * 2
    value = kv_bytes / secs / 1e9
    sample = (f"{count} requests of config 5 per step (lengths {int(lens.min())}..{int(lens.max())}), "
              f"gather + reference_attention, one request per thread")
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": secs * 1e3, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "config5 decode (Llama-3-70B heads 64Q/8KV hd128 bf16), CPU sample",
                       "global_batch": cfg["batch"], "seq_len": "U[4096,32768]", "parallelism": "host threads"},
            "cpu_baseline": {"value": value, "unit": "GB/s", "cores": threads, "kind": kind, "sample": sample},
            "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------- single case ---

def only_case(args, ranks: Ranks, kv, w, peak: float) -> int:
    """One kernel's case on its own (used under ncu): setup, `warmup` untimed
    launches, `steps` timed launches, one short JSON line."""
    import torch

    if args.only in ("decode5", "decode3"):
        cfg = dict(w.CONFIG5 if args.only == "decode5" else w.CONFIG3)
        if args.batch:
            cfg["batch"] = args.batch
        if args.pps:
            cfg["pages_per_split"] = args.pps
        # --shard N: rank 0's KV-head shard of an N-way split, on this one GPU
        # (every rank's shard has the same shape; only the seeds differ).
        shard_world = args.shard or ranks.world
        wl = Decode(kv, w, cfg, ranks.rank, shard_world)
        per, total = time_launches(wl.launch, args.steps, args.warmup, ranks)
        ms = total / args.steps
        out = {"case": args.only, "batch": cfg["batch"], "shard_of": shard_world, "ms_per_launch": ms,
               "kv_bytes": wl.kv_bytes, "algorithmic_bytes": wl.alg_bytes,
               "gbs": wl.alg_bytes / (ms * 1e-3) / 1e9, "pages_per_split": wl.pps}
    elif args.only == "step5":
        cfg = dict(w.CONFIG5)
        if args.batch:
            cfg["batch"] = args.batch
        wl = Decode(kv, w, cfg, ranks.rank, ranks.world)
        out = decode_step(kv, wl, args.steps, args.warmup, ranks)
        out.update({"case": args.only, "batch": cfg["batch"], "gbs": out["fused_kv_gbs"]})
    elif args.only == "layers":
        out = layer_batches(kv, w, ranks.rank, ranks.world, ranks, layers=args.batch or 32, steps=args.steps,
                            warmup=args.warmup, graph=args.steps >= 10, tokens=args.tokens or 1024)
        out.update({"case": args.only, "gbs": out["gather_gbs"]})
    elif args.only == "prefill4":
        pf = Prefill(kv, w, w.CONFIG4)
        per, total = time_launches(pf.launch_batch, args.steps, args.warmup, ranks)
        ms = total / args.steps
        per1, total1 = time_launches(pf.launch, args.steps, args.warmup, ranks)
        out = {"case": args.only, "ms_per_step": ms, "launches_per_step": 1,
               "per_sequence_calls_ms_per_step": total1 / args.steps,
               "tflops": pf.flops / (ms * 1e-3) / 1e12, "gbs": 0.0}
        out["frac_of_bf16_peak"] = out["tflops"] / load_bf16_peak()[0]
    elif args.only in ("write", "gather"):
        cfg = dict(w.CONFIG2)
        if args.batch:  # fewer sequences on a proportionally smaller pool
            cfg["pool_pages"] = max(1, cfg["pool_pages"] * args.batch // cfg["sequences"])
            cfg["sequences"] = args.batch
        wg = WriteGather(kv, w, cfg, ranks.rank, ranks.world)
        fn = wg.write if args.only == "write" else wg.gather
        per, total = time_launches(fn, args.steps, args.warmup, ranks)
        ms = total / args.steps
        nbytes = wg.write_bytes if args.only == "write" else wg.gather_bytes
        out = {"case": args.only, "ms_per_launch": ms, "algorithmic_bytes": nbytes,
               "gbs": nbytes / (ms * 1e-3) / 1e9}
    else:  # gather_tma, gather_ldst
        cfg = dict(w.CONFIG2)
        if args.batch:  # fewer sequences on a proportionally smaller pool
            cfg["pool_pages"] = max(1, cfg["pool_pages"] * args.batch // cfg["sequences"])
            cfg["sequences"] = args.batch
        wg = WriteGather(kv, w, cfg, ranks.rank, ranks.world)
        tma = args.only == "gather_tma"
        per, total = time_launches(lambda st: wg.gather_one_by_one(st, tma), args.steps, args.warmup, ranks)
        ms = total / args.steps
        out = {"case": args.only, "ms_per_step": ms, "sequences": wg.nseq, "algorithmic_bytes": wg.gather_bytes,
               "gbs": wg.gather_bytes / (ms * 1e-3) / 1e9}
    out["frac_of_peak"] = out["gbs"] / peak
    torch.cuda.synchronize()
    if ranks.rank == 0:
        print(json.dumps(out), flush=True)
    ranks.close()
    return 0


# ------------------------------------------------------------------- main ---

def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-secondary", action="store_true", help="headline decode only")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--only", choices=["decode5", "decode3", "write", "gather", "gather_tma", "gather_ldst",
                                       "prefill4", "step5", "layers"],
                    help="run one kernel's case alone (profiling runs); prints a short JSON line")
    ap.add_argument("--batch", type=int, default=None, help="override the batch: decode requests, write/gather sequences (profiling runs)")
    ap.add_argument("--shard", type=int, default=None,
                    help="with --only decode5/decode3 on one GPU: time rank 0's shard of an N-way KV-head split")
    ap.add_argument("--tokens", type=int, default=None,
                    help="with --only layers: tokens per sequence (the pool shrinks with it; profiling runs)")
    ap.add_argument("--pps", type=int, default=None,
                    help="with --only decode5/decode3: pages per split instead of the library's choice")
    args = ap.parse_args(argv)
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    ranks = Ranks(args.gpus)
    if args.impl == "reference":
        return reference_arm(args, ranks)

    import torch

    import kvflux_b200 as kv
    from kvflux_b200 import workloads as w

    ranks.init_gpu()
    world, rank = ranks.world, ranks.rank
    peak, peak_kind = load_peak()
    if args.only:
        return only_case(args, ranks, kv, w, peak)

    wl = Decode(kv, w, w.CONFIG5, rank, world)
    pps5 = wl.pps
    clk = Clocks(ranks.local).__enter__()
    per, total_ms = time_launches(wl.launch, args.steps, args.warmup, ranks)
    ms = ranks.reduce(total_ms / args.steps, "max")
    kv_bytes_all = ranks.reduce(float(wl.kv_bytes), "sum")
    value = kv_bytes_all / (ms * 1e-3) / 1e9
    kernel_ms = statistics.mean(per)
    achieved = wl.alg_bytes / (kernel_ms * 1e-3) / 1e9
    ratio, capture = traffic_ratio("decode_mma_kernel")
    roofline = {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                "peak_kind": peak_kind, "traffic": (ratio * wl.alg_bytes) if ratio else None,
                "traffic_source": capture, "algorithmic_bytes_per_launch": wl.alg_bytes,
                "kernel_ms_per_launch": kernel_ms, "frac_of_datasheet": achieved / DATASHEET_GBS}

    # Outputs of all ranks to rank 0 over NCCL, for verification only (outside the timed region).
    finite = bool(torch.isfinite(wl.o).all().item())
    if ranks.dist is not None:
        gathered = [torch.empty_like(wl.o) for _ in range(world)]
        ranks.dist.all_gather(gathered, wl.o)
        if rank == 0:
            full = torch.stack([g.view(wl.batch, wl.qh, wl.hd) for g in gathered], dim=1)
            finite = bool(torch.isfinite(full).all().item()) and full.shape[1] * full.shape[2] == w.CONFIG5["q_heads"]
        del gathered

    e2e_ms, h2d, d2h_bytes, dev_api_ms = e2e_decode(kv, wl, max(3, args.steps // 4), 3)
    clk.__exit__(None, None, None)
    e2e_ms = ranks.reduce(e2e_ms, "max")
    dev_api_ms = ranks.reduce(dev_api_ms, "max")
    e2e = {"value": kv_bytes_all / (e2e_ms * 1e-3) / 1e9, "unit": "GB/s", "ms_per_step": e2e_ms,
           "h2d_bytes_per_step": h2d * world, "d2h_bytes_per_step": d2h_bytes * world,
           "api": "kvflux::v2::paged_attention_batch_host (pinned host Q in, O out)",
           "device_api": {"api": "Q H2D + kvflux::v2::paged_attention_batch + O D2H", "ms_per_step": dev_api_ms,
                          "value": kv_bytes_all / (dev_api_ms * 1e-3) / 1e9}}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        sample_req = list(range(min(16, wl.batch)))
        hk, hv, nb, table, lens, q, o_gpu = wl.host_sample(sample_req)
        gbs, secs, kind, cores, count, out, one_core = cpu_decode_sample(hk, hv, nb, wl.kvh, wl.bs, wl.hd, table,
                                                                         lens, wl.qh, q)
        err = float(np.abs(out[:count * wl.qh * wl.hd] - o_gpu[:count * wl.qh * wl.hd]).max())
        cpu = {"value": gbs, "unit": "GB/s", "cores": cores, "kind": kind,
               "sample": f"{count} of config 5's 256 requests (gather + reference_attention), {secs:.1f} s",
               "max_abs_err_vs_gpu": err,
               "single_core": {"value": one_core, "unit": "GB/s", "cores": 1,
                               "sample": "request 0 alone, the same code on one thread"},
               # The reference's own GPU kernels on this box, beside this build's.
               "reference_gpu_kernels": reference_gpu_sample(kv, w)}

    secondary = {}
    if not args.no_secondary:
        # Mutates the sequences (one token per step) and wl.o: after the CPU leg.
        secondary["decode_step_cfg5"] = decode_step(kv, wl, max(3, args.steps // 2), 3, ranks)
        del wl
        torch.cuda.empty_cache()
        wg = WriteGather(kv, w, w.CONFIG2, rank, world)
        per_w, tot_w = time_launches(wg.write, 50, 5, ranks)
        w_ms = ranks.reduce(tot_w / 50, "max")
        g_ms_launch = ranks.reduce(wg.graph_write_ms(), "max")
        e2e_w_ms, e2e_w_h2d = wg.e2e_write_ms()
        e2e_w_ms = ranks.reduce(e2e_w_ms, "max")
        write_bytes_all = ranks.reduce(float(wg.write_bytes), "sum")
        per_g, tot_g = time_launches(wg.gather, 10, 3, ranks)
        g_ms = ranks.reduce(tot_g / 10, "max")
        gather_bytes_all = ranks.reduce(float(wg.gather_bytes), "sum")
        secondary["kv_write"] = {
            "workload": "config2 write: 256 new tokens (64 seqs x 4) per step, 8 KV heads x 128, bf16, odd/even pool",
            "tokens_per_s": wg.n / (w_ms * 1e-3), "ms_per_launch": w_ms,
            "graph_tokens_per_s": wg.n / (g_ms_launch * 1e-3), "graph_ms_per_launch": g_ms_launch,
            "graph_hbm_gbs": write_bytes_all / (g_ms_launch * 1e-3) / 1e9,
            "graph_frac_of_peak": write_bytes_all / (g_ms_launch * 1e-3) / 1e9 / (peak * world),
            "e2e_tokens_per_s": wg.n / (e2e_w_ms * 1e-3), "e2e_h2d_bytes_per_step": e2e_w_h2d * world,
            "l2": f"timed launches rotate over {wg.rot} slot/input sets "
                  f"({wg.rot * wg.write_bytes / 1e6:.0f} MB touched per rotation, L2 126 MB)"}
        secondary["gather"] = {
            "workload": "config2 gather: 64 seqs x 8192 tokens to contiguous K/V, one kvfx_gather_batch launch",
            "gbs": gather_bytes_all / (g_ms * 1e-3) / 1e9, "ms_per_step": g_ms,
            "frac_of_peak": gather_bytes_all / (g_ms * 1e-3) / 1e9 / (peak * world)}
        del wg
        torch.cuda.empty_cache()
        w3 = Decode(kv, w, w.CONFIG3, rank, world)
        per3, tot3 = time_launches(w3.launch, args.steps, args.warmup, ranks)
        ms3 = ranks.reduce(tot3 / args.steps, "max")
        kv3 = ranks.reduce(float(w3.kv_bytes), "sum")
        alg3 = ranks.reduce(float(w3.alg_bytes), "sum")
        secondary["decode_cfg3"] = {
            "workload": "config3 decode: Llama-3-8B heads 32Q/8KV hd128 bf16, batch 64, L~U[512,8192]",
            "kv_gbs": kv3 / (ms3 * 1e-3) / 1e9, "ms_per_step": ms3,
            "frac_of_peak": alg3 / (ms3 * 1e-3) / 1e9 / (peak * world)}
        del w3
        torch.cuda.empty_cache()
        secondary["layers_cfg2"] = layer_batches(kv, w, rank, world, ranks)
        torch.cuda.empty_cache()
        if rank == 0:
            pf = Prefill(kv, w, w.CONFIG4)
            per4, tot4 = time_launches(pf.launch_batch, 3, 3, Ranks.this_rank_only())
            ms4 = tot4 / 3
            _, tot4s = time_launches(pf.launch, 3, 3, Ranks.this_rank_only())
            bf16_peak, bf16_kind = load_bf16_peak()
            secondary["prefill_cfg4"] = {
                "workload": "config4 causal prefill: 8 x 4096 tokens, 32Q/8KV hd128 bf16, sequences 0-3 share 2056 "
                            "tokens (partial page copy-on-written), tcgen05 kernel",
                "ms_per_step": ms4, "launches_per_step": 1, "api": "kvfx_attention_batch",
                "per_sequence_calls_ms_per_step": tot4s / 3, "cow_page_copies": pf.cow_copies,
                "algorithmic_tflops": pf.flops / (ms4 * 1e-3) / 1e12,
                "frac_of_bf16_peak": pf.flops / (ms4 * 1e-3) / 1e12 / bf16_peak, "peak_kind": bf16_kind,
                "tensor_flops_executed_per_algorithmic": 2.0}
            del pf

    clocks = clk.summary()
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded N(0,1) bf16 K/V, FP32 Q)",
            "config": {"workload": "config5 decode: Llama-3-70B heads 64Q/8KV hd128 bf16, batch 256, "
                                   "L~U[4096,32768], block 16, random-fragmented pools, KV heads sharded over ranks",
                       "global_batch": w.CONFIG5["batch"], "seq_len": "U[4096,32768]",
                       "parallelism": f"kv-head shard x{world}", "l2": "inputs larger than L2 (no flush)",
                       "pages_per_split": pps5},
            "frac_of_measured_hbm": value / (peak * world), "frac_of_datasheet_hbm": value / (DATASHEET_GBS * world),
            "roofline": roofline, "e2e": e2e, "cpu_baseline": cpu, "gpu_launches": args.steps,
            "clocks": clocks, "outputs_finite": finite, "secondary": secondary,
        }
        print(json.dumps(line), flush=True)
    ranks.close()
    return 0


if __name__ == "__main__":
    sys.exit(main())
