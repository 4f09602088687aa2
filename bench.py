"""Benchmark: batched TT-KV decode step on Llama-3.2-3B-shaped layers.

One STEP = for each of the 28 layers: encode the step's new token of every request into its slot
(frozen projection + residual/V select-pack in one clustered launch, `ttkv_write_paged`) and read
every request's whole store (`ttkv_decode_paged`: reconstruct, patch, rotate, score, online
softmax, V readout). Each layer's launches are replayed from a CUDA graph (`--no-graph`: eager).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Prints ONE JSON line (rank 0). `value` = decoded tokens/s of the whole job (requests x ranks /
step time, device-timed, max over ranks). Inputs are synthetic (seeded; shapes of config 1) and
the stores are encoded by this repository's own encoder (device TT-SVD fit per request and
layer, then the CUDA writer). The per-step working set (~0.9 GB of slots) exceeds L2, so no flush
is needed between steps.

Multi-GPU (torchrun): KV heads are sharded across ranks for the read (rank g stores and reads heads
[g*H/N, (g+1)*H/N) of every request, the storage-sharded format) and every rank ends each layer
with every head of the output: by default the decode's merge stores its rows into every rank's
output over NVLink peer memory and the step waits on the device for the other ranks' rows
(`--gather p2p`, no collective per layer), or through an NCCL all-gather per layer (`--gather
nccl`). The write's projection is replicated (every rank projects the step's tokens, then packs
its own heads). Total work is fixed as N grows ("strong").
"""
from __future__ import annotations

import argparse
import json
import os
import pathlib
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = pathlib.Path(__file__).resolve().parent
for _p in (ROOT, ROOT / "ttkv-vllm_b200"):
    if str(_p) not in sys.path:
        sys.path.insert(0, str(_p))

METRIC = "decode step ms & tok/s (3B shape, bs1-64, 1k-16k ctx) + HBM GB/s vs peak"

# DRAM bytes (read + write) of ONE decode launch from an ncu capture of this workload's layer 9
# (r1 = 110, 8 requests x 4323 rows), and a hash of the read kernel's sources at the time of the
# capture. The per-launch `traffic` of the roofline scales it by algorithmic bytes (the kernel reads
# each slot byte once, so traffic grows in proportion to the rows and widths a launch reads); when
# the sources no longer hash the same, the capture describes another kernel and `traffic` is null.
CAPTURED_LAUNCH = {"layer": 9, "dram_bytes": 37336320, "src_sha16": "9a6dec30c44e4a5e",
                   "kernel": "decode_tc_kernel<3, bf16 table>"}
READ_SOURCES = ("ttkv-vllm_b200/csrc/ttkv_read.cu", "ttkv-vllm_b200/csrc/ttkv_decode_tc.cuh")


def read_src_sha16() -> str:
    import hashlib
    h = hashlib.sha256()
    for f in READ_SOURCES:
        h.update((ROOT / f).read_bytes())
    return h.hexdigest()[:16]


def _peaks():
    """(HBM GB/s, bf16 TFLOP/s burst, bf16 TFLOP/s sustained, "measured" | "fallback")."""
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return (float(d["hbm_gbs"]), float(d["bf16_tflops"]),
                float(d.get("bf16_tflops_sustained", d["bf16_tflops"])), "measured")
    return 6650.0, 1590.0, 1400.0, "fallback"


# ---------------------------------------------------------------------------- clocks
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except (FileNotFoundError, OSError):
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if self.proc is None or not self.path:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        rows = []
        for line in pathlib.Path(self.path).read_text().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) >= 9:
                rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons, "samples": len(rows)}


# ---------------------------------------------------------------------------- workload
def synth_kv_device(gen, H, n, d=128, rank=96, dtype=None):
    """Device version of vllm_ttkv.synthetic.synth_kv's distribution (seeded torch generator)."""
    import torch
    dev = gen.device
    Z = torch.randn(H, n, rank, generator=gen, device=dev)
    B = torch.randn(H, rank, d, generator=gen, device=dev) / rank ** 0.5
    idx = torch.stack([torch.randperm(d, generator=gen, device=dev)[:4] for _ in range(H)])
    scale = torch.ones(H, 1, d, device=dev)
    scale.scatter_(2, idx.unsqueeze(1), 8.0)
    K = torch.bmm(Z, B * scale) + 0.02 * torch.randn(H, n, d, generator=gen, device=dev)
    V = torch.randn(H, n, d, generator=gen, device=dev)
    if dtype is not None:
        K, V = K.to(dtype), V.to(dtype)
    return K, V


class Workload:
    """Config-1 stores on one device: per layer a paged cache, a decoder pool and pinv pool."""

    def __init__(self, B, n, r1s, cfg, device, dtype, seed=0, block_size=16, HQ=24, H=8):
        import numpy as np
        import torch

        from vllm_ttkv import encode, ops, synthetic
        from vllm_ttkv.layout import layout_for_config
        self.B, self.n, self.HQ, self.H, self.bs = B, n, HQ, H, block_size
        self.r1s = list(r1s)
        self.L = len(self.r1s)
        self.device, self.dtype = device, dtype
        seq = n + 1                                            # the stored rows incl. this step's
        bt_np, n_blocks = synthetic.block_table(seed, [seq] * B, block_size)
        self.block_table = torch.from_numpy(bt_np).to(device)
        self.seq_lens = torch.full((B,), seq, dtype=torch.int32, device=device)
        self.max_seq = seq
        self.n_slots = n_blocks * block_size
        slots_all = torch.from_numpy(
            (bt_np[:, :, None].astype(np.int64) * block_size + np.arange(block_size)
             ).reshape(B, -1)[:, :seq]).to(device)
        self.new_slots = slots_all[:, n].contiguous()             # [B] slot of the step's token
        gen = torch.Generator(device=device)
        gen.manual_seed(seed)
        self.layouts, self.caches, self.decoders, self.pinvT, self.images = [], [], [], [], []
        self.k_new, self.v_new, self.q, self.out = [], [], [], []
        self.fit_s = 0.0
        self.dec_index = torch.arange(B, dtype=torch.int32, device=device)
        # every layer's step inputs (q, the new token's K and V) in one device buffer and every
        # layer's output in another, so a step's host transfers are one copy each way
        per_in = B * (HQ + 2 * H) * 128
        self.inbuf = torch.empty(self.L * per_in, dtype=dtype, device=device)
        self.outbuf = torch.empty(self.L * B * HQ * 128, dtype=dtype, device=device)
        for l, r1 in enumerate(self.r1s):
            lay = layout_for_config(cfg, r1, H=H)
            cache = torch.zeros(self.n_slots, lay.compressed_bytes_per_token(), dtype=torch.uint8,
                                device=device)
            dec = torch.zeros(B, r1, H * 128, device=device)
            pinvT = torch.zeros(B, r1, H * 128, device=device)
            base = l * per_in
            qv = self.inbuf[base:base + B * HQ * 128].view(B, HQ, 128)
            kn = self.inbuf[base + B * HQ * 128:base + B * (HQ + H) * 128].view(B, H, 128)
            vn = self.inbuf[base + B * (HQ + H) * 128:base + per_in].view(B, H, 128)
            for r in range(B):
                K, V = synth_kv_device(gen, H, seq, dtype=dtype)
                t0 = time.perf_counter()
                fk = encode.fit_into_budget(K[:, :n], lay, cfg)
                encode.write_fitted(cache, slots_all[r, :n].contiguous(), fk,
                                    K[:, :n].permute(1, 0, 2).contiguous(),
                                    V[:, :n].permute(1, 0, 2).contiguous(), lay)
                dec[r] = fk.decoder.decoder_f
                pinvT[r] = fk.decoder.pinvT
                torch.cuda.synchronize(device)
                self.fit_s += time.perf_counter() - t0
                kn[r] = K[:, n].to(dtype)
                vn[r] = V[:, n].to(dtype)
            self.layouts.append(lay)
            self.caches.append(cache)
            self.decoders.append(dec)
            self.images.append(ops.decoder_image(lay, dec))       # made once per decoder, as the pool does
            self.pinvT.append(pinvT)
            self.k_new.append(kn)
            self.v_new.append(vn)
            qv.copy_(torch.randn(B, HQ, 128, generator=gen, device=device))
            self.q.append(qv)
            self.out.append(self.outbuf[l * B * HQ * 128:(l + 1) * B * HQ * 128].view(B, HQ, 128))
        self.heads = (0, H)
        self.peers = None                      # per layer ttkv_peers_t of a fused gather (PeerGather)
        self.read_layouts = list(self.layouts)
        self.read_dec = list(self.decoders)
        self.table = torch.from_numpy(synthetic.cos_sin_cache(seq + 16, dtype="float32")).to(device).to(dtype)
        self.scale = 128 ** -0.5

    def shard(self, lo, hi):
        """Keep only KV heads [lo, hi) in storage, the storage-sharded format of tensor
        parallelism: each layer's cache becomes the blobs of `lay.shard(lo, hi)` (the coefficient
        block and these heads' rows), the read's decoders these heads' columns. The write still
        projects every head (the pinv and K of all heads), and packs these heads only."""
        from vllm_ttkv import ops
        from vllm_ttkv.layout import shard_slots
        self.heads = (lo, hi)
        for l in range(self.L):
            lay = self.layouts[l]
            self.caches[l] = shard_slots(self.caches[l], lay, lo, hi)
            self.read_layouts[l] = lay.shard(lo, hi)
            self.read_dec[l] = self.decoders[l][:, :, lo * 128:hi * 128].contiguous()
            self.images[l] = ops.decoder_image(self.read_layouts[l], self.read_dec[l])
        import torch
        torch.cuda.empty_cache()

    def slot_bytes(self, l):
        return self.B * self.max_seq * self.read_layouts[l].compressed_bytes_per_token()

    def read_bytes(self, l):
        """Algorithmic bytes of one decode launch: the slots (this rank's storage: the coefficient
        block and its heads' rows), the decoders (fp32, the heads read), the queries and outputs."""
        lay = self.read_layouts[l]
        dec = self.B * lay.r1 * lay.H * 128 * 4
        io = 2 * self.B * (self.HQ * lay.H // self.H) * 128 * 2
        return self.B * self.max_seq * lay.compressed_bytes_per_token() + dec + io

    def write(self, l):
        """The write of the step's token of every request (every head projected; this rank's
        heads packed)."""
        from vllm_ttkv import encode
        encode.write_frozen(self.caches[l], self.new_slots, self.k_new[l], self.v_new[l],
                            self.dec_index, self.decoders[l], self.pinvT[l], self.layouts[l],
                            heads=self.heads)

    def read(self, l):
        """The read of every request's store: this rank's query heads of out[l]."""
        from vllm_ttkv import ops
        lo, hi = self.heads
        G = self.HQ // self.H
        ops.decode_paged(self.read_layouts[l], self.caches[l], self.bs, self.block_table, self.seq_lens,
                         self.read_dec[l], self.dec_index, self.table, self.q[l][:, lo * G:hi * G],
                         self.scale, self.out[l][:, lo * G:hi * G], self.max_seq, images=self.images[l],
                         peers=self.peers[l] if self.peers else None)

    def layer_step(self, l):
        """One layer: write the step's token of every request, then read every request's store."""
        self.write(l)
        self.read(l)


# ---------------------------------------------------------------------------- plugin e2e
def plugin_e2e(wl, steps, warmup, device, graph=False):
    """The step through the reference-facing plugin, `TTKVAttentionImpl.forward`, once per layer:
    the raw key handed over by the rotary capture's stash; every layer's q/k/v copied in from
    pinned host memory (one copy) and every layer's output copied back (one copy).

    eager: one new metadata object (and host-read step plan) per step, forward per layer.
    graph: the 28 forward calls captured once in one CUDA graph (the device-planned decode step:
    pool rows looked up on the device, no readback) and replayed per step, as an engine that
    captures decode steps does; the copies in and out stay outside the graph, every step.
    Returns (ms per step, h2d bytes, d2h bytes)."""
    from types import SimpleNamespace

    import torch

    from vllm_ttkv import encode, metadata, ops, patch, rope_store
    from vllm_ttkv.impl import TTKVAttentionImpl
    impl = TTKVAttentionImpl(wl.HQ, 128, wl.scale, wl.H)
    keys = [int(x) for x in wl.block_table[:, 0].tolist()]
    layers = []
    for l in range(wl.L):
        lay = wl.layouts[l]
        layer = SimpleNamespace(layer_name=f"model.layers.{l}.self_attn.attn", ttkv_layout=lay,
                                rotary_emb=SimpleNamespace(cos_sin_cache=wl.table))
        for r in range(wl.B):
            kd = encode.KDecoder(wl.decoders[l][r])
            kd._pinvT = wl.pinvT[l][r]
            rope_store.register_decoder(layer.layer_name, keys[r], kd, lay=lay)
        page = wl.caches[l].view(-1, 1, wl.bs, wl.caches[l].shape[1])
        layers.append((layer, page))
    pin_in = wl.inbuf.cpu().pin_memory()                 # every layer's q, K, V of the step
    pin_o = torch.empty(wl.outbuf.shape, dtype=wl.outbuf.dtype).pin_memory()
    h2d = pin_in.numel() * pin_in.element_size()
    d2h = pin_o.numel() * pin_o.element_size()
    qsl_cpu = torch.arange(wl.B + 1, dtype=torch.int32)
    qsl = qsl_cpu.to(device)

    def new_md():
        return metadata.TTKVAttentionMetadata(
            seq_lens=wl.seq_lens, slot_mapping=wl.new_slots, block_table=wl.block_table,
            query_start_loc=qsl, query_start_loc_cpu=qsl_cpu, num_actual_tokens=wl.B,
            max_query_len=1, max_seq_len=wl.max_seq, ttkv_serial=metadata.next_serial())

    def forward(l, md):
        layer, page = layers[l]
        patch.stash_raw_k(layer.layer_name, wl.k_new[l], None, wl.table)
        impl.forward(layer, wl.q[l], None, wl.v_new[l], page, md, wl.out[l])

    if graph:
        md = new_md()
        ops.status_word(device)
        side = torch.cuda.Stream(device)
        side.wait_stream(torch.cuda.current_stream(device))
        with torch.cuda.stream(side):              # eager warm-up: workspaces, key map, pools
            for l in range(wl.L):
                forward(l, md)
        torch.cuda.current_stream(device).wait_stream(side)
        torch.cuda.synchronize(device)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for l in range(wl.L):
                forward(l, md)

        def step():
            wl.inbuf.copy_(pin_in, non_blocking=True)
            g.replay()
            pin_o.copy_(wl.outbuf, non_blocking=True)
    else:
        def step():
            md = new_md()
            wl.inbuf.copy_(pin_in, non_blocking=True)
            for l in range(wl.L):
                forward(l, md)
            pin_o.copy_(wl.outbuf, non_blocking=True)

    for _ in range(warmup):
        step()
    torch.cuda.synchronize(device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        step()
    e1.record()
    torch.cuda.synchronize(device)
    ops.check_status(device)
    if graph:
        del g
    rope_store.clear_decoders()
    rope_store.clear_stores()
    return e0.elapsed_time(e1) / steps, h2d, d2h


# ---------------------------------------------------------------------------- CPU baseline
def cpu_sample(wl_params, sample_layers=(0, 9, 18, 27), reps=1, seed=0):
    """Time the oracle (the reference's torch CPU path restated in numpy) on a bounded sample of
    (request, layer) pairs of the same workload, built on the CPU by the oracle's own fit:
    a decode read over n+1 rows plus the write of one token. Returns seconds per (request, layer)
    averaged over the sample."""
    import numpy as np

    from oracle import ttkv_oracle as O
    from vllm_ttkv import synthetic as S
    B, n, r1s, cfg = wl_params
    per = []
    for i, l in enumerate(sample_layers):
        g = O.geometry_for_config(cfg, r1s[l])
        K, V = S.synth_kv(seed + i, n + 1)
        f = O.fit_into_budget(K[:, :n], g, cfg)
        blobs = O.build_slots(g, f["coeff_q"], f["coeff_scale"], f["R"], V[:, :n])
        pinv = np.linalg.pinv(f["decoder_f"]).astype(np.float32)
        table = S.cos_sin_cache(n + 16, dtype="bfloat16")
        q = S.synth_queries(seed + i, (24, 128), "bfloat16")
        cos, sin = O.cos_sin_from_table(table, np.arange(n + 1), 128)
        t0 = time.perf_counter()
        for _ in range(reps):
            cq, cs, R = O.encode_frozen(K[:, n:n + 1], f["decoder_f"], pinv)
            blob = O.build_slots(g, cq, cs, R, V[:, n:n + 1])
            allb = np.concatenate([blobs, blob])
            O.attend(g, allb[:, :g.k_slot_bytes], allb[:, g.k_slot_bytes:], f["decoder_f"], q, cos, sin)
        per.append((time.perf_counter() - t0) / reps)
    return sum(per) / len(per)


SAMPLE_LAYERS = (0, 9, 18, 27)          # the CPU sample's layers: r1 = 14, 110, 125, 67


def run_reference(args):
    """The reference arm: the reference's CPU path (the oracle's numpy port, BLAS on every host
    thread) on a bounded sample of the same workload. Step k times one (request, layer) pair --
    a write of the step's token and the read of the request's whole store -- at layer
    SAMPLE_LAYERS[k % 4]; `ms_per_step` is that measured sample, and `value` extrapolates the mean
    per-pair time to the full step (B requests x 28 layers), the factor named in the config."""
    from vllm_ttkv import synthetic as S
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    cores = os.cpu_count()
    B, n = args.batch, args.ctx
    r1s = S.LLAMA32_3B_R1
    for k in range(args.warmup):
        cpu_sample((B, n, r1s, "safe"), sample_layers=(SAMPLE_LAYERS[k % 4],), seed=100 + k)
    times = []
    for k in range(args.steps):
        times.append(cpu_sample((B, n, r1s, "safe"), sample_layers=(SAMPLE_LAYERS[k % 4],), seed=k))
    per_pair = statistics.mean(times)
    factor = B * len(r1s)
    v = B / (per_pair * factor)
    line = {"metric": METRIC, "value": v, "unit": "tok/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": per_pair * 1e3, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "impl": "reference",
            "config": {"workload": f"cfg1 decode step: B={B} x {n} ctx, 28 layers, safe; each timed step is "
                                   f"ONE (request, layer) pair cycling layers {list(SAMPLE_LAYERS)}, value "
                                   f"extrapolated x{factor} (B x 28 layers)",
                       "batch": B, "ctx": n, "layers": len(r1s), "extrapolation_factor": factor,
                       "sample_layers": list(SAMPLE_LAYERS)},
            "cpu_baseline": {"value": v, "unit": "tok/s", "cores": cores, "kind": "port",
                             "sample": f"1 (request, layer) pair per step at n={n}, layers "
                                       f"{list(SAMPLE_LAYERS)} in turn (r1 {[r1s[l] for l in SAMPLE_LAYERS]}), "
                                       f"scaled x{factor} to a full step"},
            "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line))


# ---------------------------------------------------------------------------- other workloads
def _event_ms(fn, steps, warmup):
    import torch
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / steps


def run_prefill(args):
    """Config 3, chunked-prefill continuation: `--batch` prompts of `--prompt-len` tokens continued
    in `--chunk`-token chunks against one layer's compressed store (r1 = 110, `safe`, fp16 store,
    block 16). One step = every chunk after the first: the frozen write of the chunk's tokens of all
    prompts, then ONE continuation read (`ttkv_prefill_cont_paged`) of all prompts, causal over the
    stored rows. The first chunk (SDPA over the model's own keys + the fit) is set-up."""
    import numpy as np
    import torch

    from vllm_ttkv import encode, ops, synthetic
    from vllm_ttkv.layout import layout_for_config
    device = torch.device("cuda", 0)
    B, N, Q, H, HQ, bs, r1 = args.batch, args.prompt_len, args.chunk, 8, 24, 16, 110
    lay = layout_for_config("safe", r1, H=H)
    bt_np, n_blocks = synthetic.block_table(0, [N] * B, bs)
    bt = torch.from_numpy(bt_np).to(device)
    slots_all = torch.from_numpy((bt_np[:, :, None].astype(np.int64) * bs + np.arange(bs)).reshape(B, -1)[:, :N]).to(device)
    cache = torch.zeros(n_blocks * bs, lay.compressed_bytes_per_token(), dtype=torch.uint8, device=device)
    gen = torch.Generator(device=device)
    gen.manual_seed(0)
    dec = torch.zeros(B, r1, H * 128, device=device)
    pinvT = torch.zeros_like(dec)
    Ks, Vs = [], []
    for r in range(B):
        K, V = synth_kv_device(gen, H, N, dtype=torch.float16)
        fk = encode.fit_into_budget(K[:, :Q], lay, "safe")
        encode.write_fitted(cache, slots_all[r, :Q].contiguous(), fk, K[:, :Q].permute(1, 0, 2).contiguous(),
                            V[:, :Q].permute(1, 0, 2).contiguous(), lay)
        dec[r], pinvT[r] = fk.decoder.decoder_f, fk.decoder.pinvT
        Ks.append(K.permute(1, 0, 2).contiguous())
        Vs.append(V.permute(1, 0, 2).contiguous())
    table = torch.from_numpy(synthetic.cos_sin_cache(N + 16, dtype="float32")).to(device).half()
    images = ops.decoder_image(lay, dec)                       # made once per decoder, as the pool does
    q = torch.randn(B * Q, HQ, 128, generator=gen, device=device).half()
    out = torch.empty_like(q)
    idx = torch.arange(B, dtype=torch.int32, device=device)
    chunks = []
    for s0 in range(Q, N, Q):
        e = min(N, s0 + Q)
        ql = e - s0
        chunks.append(dict(
            e=e, ql=ql, slots=slots_all[:, s0:e].reshape(-1).contiguous(),
            k=torch.cat([Ks[r][s0:e] for r in range(B)]), v=torch.cat([Vs[r][s0:e] for r in range(B)]),
            tok=torch.repeat_interleave(idx, ql), seq=torch.full((B,), e, dtype=torch.int32, device=device),
            q_start=(idx * ql).contiguous(), q_len=torch.full((B,), ql, dtype=torch.int32, device=device)))
    def step():
        for c in chunks:
            encode.write_frozen(cache, c["slots"], c["k"], c["v"], c["tok"], dec, pinvT, lay)
            ops.prefill_cont_paged(lay, cache, bs, bt, c["seq"], dec, idx, table, c["q_start"], c["q_len"],
                                   q, 128 ** -0.5, out, c["ql"], c["e"], images=images)

    for _ in range(args.warmup):                               # a profiler run with
        step()                                                 # --profile-from-start off sees
    torch.cuda.synchronize()                                   # the timed steps only
    torch.cuda.cudart().cudaProfilerStart()
    ms = _event_ms(step, args.steps, 0)
    torch.cuda.cudart().cudaProfilerStop()
    # the continuation launches alone, on the launching stream
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in chunks]
    torch.cuda.synchronize()
    for (a, b), c in zip(evs, chunks):
        a.record()
        ops.prefill_cont_paged(lay, cache, bs, bt, c["seq"], dec, idx, table, c["q_start"], c["q_len"],
                               q, 128 ** -0.5, out, c["ql"], c["e"], images=images)
        b.record()
    torch.cuda.synchronize()
    read_ms = sum(a.elapsed_time(b) for a, b in evs)
    # algorithmic work of the reads: causal QK + PV over the stored rows, reconstruction once per chunk
    flops = 0.0
    for c in chunks:
        s0 = c["e"] - c["ql"]
        pairs = c["ql"] * s0 + c["ql"] * (c["ql"] + 1) / 2
        flops += B * (4 * 128 * HQ * pairs + 2 * r1 * H * 128 * c["e"])
    hbm, tc, tc_sus, peak_kind = _peaks()
    tflops = flops / (read_ms * 1e-3) / 1e12
    line = {"metric": "chunked-prefill continuation tok/s (cfg3)", "value": B * (N - Q) / (ms * 1e-3),
            "unit": "tok/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "workload": "prefill", "dtype": "fp16 model tensors, fp32 math, u8 slots",
            "data": "synthetic",
            "config": {"workload": f"cfg3: {B} prompts x {N} tokens, chunks of {Q}, 1 layer r1={r1} safe, block {bs}",
                       "chunks": len(chunks)},
            # the reads run back to back for the whole step (tens of ms): the sustained bf16 peak
            "roofline": {"bound": "tensor", "achieved": tflops, "peak": tc_sus, "unit": "TFLOP/s",
                         "frac": tflops / tc_sus, "peak_kind": "bf16 sustained (%s)" % peak_kind,
                         "read_ms_per_step": read_ms,
                         "kernel": "cont_tc_kernel (ttkv_prefill_cont_paged: a CTA per (request, KV head, "
                                   "block of 128 (query, head) rows), S and PV on tcgen05)",
                         "algorithmic_flop_per_step": flops},
            "gpu_launches": len(chunks) * 4}
    print(json.dumps(line))


def run_ttft(args):
    """A first chunk through the plugin: one request of `--prompt-len` tokens over `--layers`
    calibrated layers (`safe`, block 16, bf16), each layer one `TTKVAttentionImpl.forward` of the
    whole prompt: the TT-SVD fit and the fitted write of its keys and values, and the attention over
    its own post-RoPE q/k/v (SDPA, a library call as in the reference), which goes out first on a
    side stream and runs under the fit. Inputs are copied in from pinned host memory and the outputs
    back every step. The dense line is the same attention alone (what a dense-cache backend does at
    prefill besides its cache copy)."""
    import torch

    from vllm_ttkv import metadata, patch, rope_store
    from vllm_ttkv import synthetic as S
    from vllm_ttkv.impl import TTKVAttentionImpl
    from vllm_ttkv.decode import attend_prefill
    from vllm_ttkv.layout import layout_for_config
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    P, L, H, HQ, d, bs = args.prompt_len, args.layers, 8, 24, 128, 16
    r1s = (S.LLAMA32_3B_R1 * ((L + 27) // 28))[:L]
    gen = torch.Generator(device=device)
    gen.manual_seed(0)
    n_blocks = (P + bs - 1) // bs
    slots = torch.arange(P, device=device, dtype=torch.int64)
    bt = torch.arange(n_blocks, device=device, dtype=torch.int32).view(1, -1)
    table = torch.from_numpy(S.cos_sin_cache(P + 16, dtype="float32")).to(device).to(torch.bfloat16)
    impl = TTKVAttentionImpl(HQ, d, d ** -0.5, H)
    layers = []
    for l in range(L):
        lay = layout_for_config("safe", r1s[l], H=H)
        layer = types_ns(layer_name=f"model.layers.{l}.self_attn.attn", ttkv_layout=lay,
                         rotary_emb=types_ns(cos_sin_cache=table))
        page = torch.zeros(n_blocks, 1, bs, lay.compressed_bytes_per_token(), dtype=torch.uint8, device=device)
        layers.append((layer, page))
    # one set of q, raw K, post-RoPE K and V (every layer fits and stores the same keys: the work
    # per layer does not depend on the values), copied in every step; the last layer's output
    # copied back
    per = P * (HQ + 3 * H) * d
    K, V = synth_kv_device(gen, H, P, dtype=torch.bfloat16)
    q = torch.randn(P, HQ, d, generator=gen, device=device).to(torch.bfloat16)
    kpost = torch.randn(P, H, d, generator=gen, device=device).to(torch.bfloat16)
    pin_in = torch.cat([q.reshape(-1), K.permute(1, 0, 2).reshape(-1), kpost.reshape(-1),
                        V.permute(1, 0, 2).reshape(-1)]).cpu().pin_memory()
    del K, V, q, kpost
    dev_in = torch.empty_like(pin_in, device=device)
    out = torch.empty(P, HQ, d, dtype=torch.bfloat16, device=device)
    pin_o = torch.empty(out.shape, dtype=out.dtype).pin_memory()

    def views(l):
        b = dev_in
        q = b[:P * HQ * d].view(P, HQ, d)
        k = b[P * HQ * d:P * (HQ + H) * d].view(P, H, d)
        kp = b[P * (HQ + H) * d:P * (HQ + 2 * H) * d].view(P, H, d)
        v = b[P * (HQ + 2 * H) * d:].view(P, H, d)
        return q, k, kp, v

    qsl_cpu = torch.tensor([0, P], dtype=torch.int32)

    def step():
        dev_in.copy_(pin_in, non_blocking=True)
        md = metadata.TTKVAttentionMetadata(
            seq_lens=torch.tensor([P], dtype=torch.int32, device=device), slot_mapping=slots,
            block_table=bt, query_start_loc=qsl_cpu.to(device), query_start_loc_cpu=qsl_cpu,
            num_actual_tokens=P, max_query_len=P, max_seq_len=P, ttkv_serial=metadata.next_serial())
        for l, (layer, page) in enumerate(layers):
            q, k, kp, v = views(l)
            patch.stash_raw_k(layer.layer_name, k, None, table)
            impl.forward(layer, q, kp, v, page, md, out)
        pin_o.copy_(out, non_blocking=True)

    def dense_step():
        for l in range(L):
            q, k, kp, v = views(l)
            out.copy_(attend_prefill(q.float(), kp.float(), v.float(), d ** -0.5))

    ms = _event_ms(step, args.steps, args.warmup)
    dense_ms = _event_ms(dense_step, args.steps, args.warmup)
    rope_store.clear_decoders()
    h2d = pin_in.numel() * 2
    line = {"metric": "first-chunk (prefill) attention + TT-KV fit and write, ms to first token",
            "value": ms, "unit": "ms", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ms, "higher_is_better": False, "workload": "ttft",
            "dtype": "bf16 model tensors, fp32 fit and attention, u8 slots", "data": "synthetic",
            "config": {"workload": f"1 request x {P} tokens, {L} calibrated layers, safe, block 16, "
                                   f"through TTKVAttentionImpl.forward (fit + write + SDPA per layer)"},
            "e2e": {"value": ms, "unit": "ms", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": pin_o.numel() * 2},
            "dense_prefill_attention_ms": dense_ms}
    print(json.dumps(line))


def types_ns(**kw):
    from types import SimpleNamespace
    return SimpleNamespace(**kw)


def run_encode(args):
    """Config 4, the write path at prefill: requests of `--prompt-len` tokens (16384 for config 4),
    `--layers` layers at the `tight` allocation with r1 = 110: per layer the TT-SVD fit (library
    calls: `torch.linalg.svd` / the Gram matrix's `eigh`) + the fit tail and the fitted write (this
    repository's kernels). The batch is split by request across ranks (torchrun: request r on rank
    r, no exchange, `vllm_ttkv.shard.request_range`); a single GPU runs one request. `value` =
    tokens of all ranks / the slowest rank's step time (weak scaling: one request per GPU)."""
    import numpy as np
    import torch
    import torch.distributed as dist

    from vllm_ttkv import encode, ops, synthetic
    from vllm_ttkv.layout import layout_for_config
    from vllm_ttkv.shard import gather_bytes, request_range
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", device_id=device, timeout=datetime.timedelta(seconds=120))
    lo, hi = request_range(rank, world, world)             # one request per GPU (weak scaling)
    n, H, r1, L = args.prompt_len, 8, 110, args.layers
    lay = layout_for_config("tight", r1, H=H)
    reqs = list(range(lo, hi))
    caches, KVs = [], []
    for r in reqs:
        gen = torch.Generator(device=device)
        gen.manual_seed(1000 + r)                      # request r's keys, whichever rank has it
        caches.append(torch.zeros(n, lay.compressed_bytes_per_token(), dtype=torch.uint8, device=device))
        KVs.append([synth_kv_device(gen, H, n, dtype=torch.bfloat16) for _ in range(min(L, 4))])
    toks = [[(K.permute(1, 0, 2).contiguous(), V.permute(1, 0, 2).contiguous()) for K, V in kv] for kv in KVs]
    slots = torch.arange(n, dtype=torch.int64, device=device)
    fits = {}

    def step():
        for i in range(len(reqs)):
            for l in range(L):
                K, _ = KVs[i][l % len(KVs[i])]
                kt, vt = toks[i][l % len(KVs[i])]
                fk = encode.fit_into_budget(K, lay, "tight")
                encode.write_fitted(caches[i], slots, fk, kt, vt, lay)
                fits[(i, l % len(KVs[i]))] = fk

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(device)
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        step()
    e1.record()
    torch.cuda.synchronize(device)
    ms_t = torch.tensor([e0.elapsed_time(e1) / args.steps], device=device)
    if world > 1:
        dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
    ms = float(ms_t.item())
    # this repository's write launch alone (the select/quantise/pack of every token), per layer
    fk = fits[(0, 0)]
    kt, vt = toks[0][0]
    w_ms = _event_ms(lambda: encode.write_fitted(caches[0], slots, fk, kt, vt, lay), 10, 3)
    # the slot bytes of every request, gathered for their checksum (the byte comparison itself is
    # tests/test_baseline_configs.py's)
    digest = None
    if world > 1:
        allb = gather_bytes(torch.cat(caches), None)
        digest = int(allb.to(torch.int64).sum().item())
        dist.barrier()
    alg = n * H * 128 * 2 * 2 + n * lay.compressed_bytes_per_token()     # K, V bf16 in; slots out
    hbm, tc, tc_sus, peak_kind = _peaks()
    gbs = alg / (w_ms * 1e-3) / 1e9
    total_req = world
    if rank == 0:
        line = {"metric": "prefill encode tok/s (cfg4, requests split across GPUs)",
                "value": total_req * n / (ms * 1e-3), "unit": f"tok/s ({L} layers)", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "ms_per_layer": ms / L,
                "higher_is_better": True, "scaling": "weak", "workload": "encode",
                "dtype": "bf16 in, fp32 fit, u8 slots", "data": "synthetic",
                "config": {"workload": f"cfg4: {total_req} request(s) x {n} tokens over {world} GPU(s) "
                                       f"(request-sharded, no exchange), {L} layers, tight r1={r1}",
                           "requests_per_rank": len(reqs), "slot_byte_sum": digest},
                "roofline": {"bound": "hbm", "achieved": gbs, "peak": hbm, "unit": "GB/s", "frac": gbs / hbm,
                             "peak_kind": peak_kind, "kernel": "encode_block_kernel (ttkv_write_paged, fit path)",
                             "write_ms_per_layer": w_ms, "alg_bytes_per_layer": alg}}
        print(json.dumps(line))
    if world > 1:
        dist.destroy_process_group()


def run_sweep(args):
    """Config 2, the long-context decode sweep: 1082 / 4322 / 8642 / 14402 cached tokens at batch
    1, 8, 32 and 64, the 28 calibrated layers at `--cfg` (campaign4x: 4-bit residual and V codes),
    block 16. One step = per layer the write of every request's new token, then the read of every
    request; the 28 layers of a step are one CUDA graph per point. Set-up fits ONE request per layer
    at the longest context (the device TT-SVD + this repository's writer) and copies its rows into
    every request's own blocks, so all requests read the same bytes from different slots (the read's
    cost depends on the layout and the lengths, not on the values). Reports each point's step time,
    and per batch the slope of step time over context (us per cached token per step)."""
    import numpy as np
    import torch

    from vllm_ttkv import encode, ops, synthetic
    from vllm_ttkv.layout import layout_for_config
    device = torch.device("cuda", 0)
    ctxs = [int(x) for x in args.sweep_ctx.split(",")]
    batches = [int(x) for x in args.sweep_batch.split(",")]
    r1s = (synthetic.LLAMA32_3B_R1 * ((args.layers + 27) // 28))[:args.layers]
    H, HQ, bs = 8, 24, 16
    Bmax, nmax = max(batches), max(ctxs) + 1
    gen = torch.Generator(device=device)
    gen.manual_seed(0)
    bt_np, n_blocks = synthetic.block_table(0, [nmax] * Bmax, bs)
    bt = torch.from_numpy(bt_np).to(device)
    slots_all = torch.from_numpy((bt_np[:, :, None].astype(np.int64) * bs + np.arange(bs))
                                 .reshape(Bmax, -1)[:, :nmax]).to(device)
    t0 = time.perf_counter()
    layers = []
    for l, r1 in enumerate(r1s):
        lay = layout_for_config(args.cfg, r1, H=H)
        cache = torch.zeros(n_blocks * bs, lay.compressed_bytes_per_token(), dtype=torch.uint8, device=device)
        K, V = synth_kv_device(gen, H, nmax, dtype=torch.bfloat16)
        fk = encode.fit_into_budget(K, lay, args.cfg)
        encode.write_fitted(cache, slots_all[0].contiguous(), fk, K.permute(1, 0, 2).contiguous(),
                            V.permute(1, 0, 2).contiguous(), lay)
        rows0 = cache[slots_all[0]]
        for r in range(1, Bmax):
            cache[slots_all[r]] = rows0
        del rows0
        dec = fk.decoder.decoder_f.unsqueeze(0).expand(Bmax, -1, -1).contiguous()
        pinvT = fk.decoder.pinvT.unsqueeze(0).expand(Bmax, -1, -1).contiguous()
        layers.append(dict(lay=lay, cache=cache, dec=dec, pinvT=pinvT, images=ops.decoder_image(lay, dec),
                           k=torch.randn(Bmax, H, 128, generator=gen, device=device).to(torch.bfloat16),
                           v=torch.randn(Bmax, H, 128, generator=gen, device=device).to(torch.bfloat16),
                           q=torch.randn(Bmax, HQ, 128, generator=gen, device=device).to(torch.bfloat16),
                           out=torch.empty(Bmax, HQ, 128, dtype=torch.bfloat16, device=device)))
    torch.cuda.synchronize(device)
    setup_s = time.perf_counter() - t0
    table = torch.from_numpy(synthetic.cos_sin_cache(nmax + 16, dtype="float32")).to(device).to(torch.bfloat16)
    dec_index = torch.arange(Bmax, dtype=torch.int32, device=device)
    hbm, tc, tc_sus, peak_kind = _peaks()
    ops.status_word(device)
    points = []
    for B in batches:
        for n in ctxs:
            seq = torch.full((B,), n + 1, dtype=torch.int32, device=device)
            new_slots = slots_all[:B, n].contiguous()

            def step():
                for L in layers:
                    encode.write_frozen(L["cache"], new_slots, L["k"][:B], L["v"][:B], dec_index[:B],
                                        L["dec"], L["pinvT"], L["lay"])
                    ops.decode_paged(L["lay"], L["cache"], bs, bt[:B], seq, L["dec"], dec_index[:B], table,
                                     L["q"][:B], 128 ** -0.5, L["out"][:B], n + 1, images=L["images"])

            step()                                     # eager once: workspaces, then one graph
            torch.cuda.synchronize(device)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                step()
            ms = _event_ms(g.replay, args.steps, args.warmup)
            del g
            alg = sum(B * (n + 1) * L["lay"].compressed_bytes_per_token()
                      + B * L["lay"].r1 * H * 128 * 4 + 2 * B * HQ * 128 * 2 for L in layers)
            points.append({"batch": B, "ctx": n, "ms_per_step": ms, "tok_s": B / (ms * 1e-3),
                           "read_gbs": alg / (ms * 1e-3) / 1e9})
    ops.check_status(device)
    slopes = {}
    for B in batches:
        pts = [p for p in points if p["batch"] == B]
        if len(pts) > 1:
            x = np.array([p["ctx"] for p in pts], float)
            y = np.array([p["ms_per_step"] for p in pts], float)
            slopes[str(B)] = float(np.polyfit(x, y, 1)[0] * 1e3)          # us per cached token
    top = max(points, key=lambda p: p["read_gbs"])
    line = {"metric": "decode step ms vs context and batch (cfg2 sweep)", "value": top["tok_s"],
            "unit": "tok/s (best point)", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
            "higher_is_better": True, "workload": "sweep", "dtype": "bf16 model tensors, fp32 math, u8 slots",
            "data": "synthetic",
            "config": {"workload": f"cfg2: ctx {ctxs} x batch {batches}, {len(layers)} calibrated layers, "
                                   f"{args.cfg}, block {bs}, one CUDA graph per step",
                       "setup_s": round(setup_s, 1)},
            "points": points, "us_per_cached_token_per_step": slopes,
            "roofline": {"bound": "hbm", "achieved": top["read_gbs"], "peak": hbm, "unit": "GB/s",
                         "frac": top["read_gbs"] / hbm, "peak_kind": peak_kind,
                         "note": "whole step (writes + reads) at the best point, algorithmic read bytes"}}
    print(json.dumps(line))


def dense_point(B, n, L, steps, warmup, device, gen, H=8, HQ=24, d=128):
    """One point of the dense comparator: L layers of one query token per request over a bf16
    [B, H, n + 1, d] K and V (torch SDPA, GQA), one CUDA graph per step."""
    import torch
    import torch.nn.functional as F
    k = [torch.randn(B, H, n + 1, d, generator=gen, device=device, dtype=torch.bfloat16) for _ in range(L)]
    v = [torch.randn(B, H, n + 1, d, generator=gen, device=device, dtype=torch.bfloat16) for _ in range(L)]
    q = [torch.randn(B, HQ, 1, d, generator=gen, device=device, dtype=torch.bfloat16) for _ in range(L)]
    out = [None] * L

    def step():
        for l in range(L):
            out[l] = F.scaled_dot_product_attention(q[l], k[l], v[l], scale=d ** -0.5, enable_gqa=True)

    step()
    torch.cuda.synchronize(device)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        step()
    ms = _event_ms(g.replay, steps, warmup)
    del g, k, v, q, out
    torch.cuda.empty_cache()
    kv = L * B * (n + 1) * H * d * 2 * 2
    return {"batch": B, "ctx": n, "ms_per_step": ms, "tok_s": B / (ms * 1e-3), "kv_gbs": kv / (ms * 1e-3) / 1e9}


def run_dense(args):
    """The dense comparator of configs 1 and 2: the same decode steps over a bf16 KV cache (4096 B
    per token per layer, what stock vLLM stores), read by torch's scaled_dot_product_attention (a
    library kernel, GQA) -- no TT-KV code. For each (batch, context) point of the sweep, one step =
    28 layers of one query token per request attending over [B, 8, n, 128] K and V, replayed from
    one CUDA graph. Reports each point's step time and its KV read rate."""
    import torch
    device = torch.device("cuda", 0)
    ctxs = [int(x) for x in args.sweep_ctx.split(",")]
    batches = [int(x) for x in args.sweep_batch.split(",")]
    L = args.layers
    gen = torch.Generator(device=device)
    gen.manual_seed(0)
    hbm, tc, tc_sus, peak_kind = _peaks()
    points = [dense_point(B, n, L, args.steps, args.warmup, device, gen) for B in batches for n in ctxs]
    top = max(points, key=lambda p: p["kv_gbs"])
    line = {"metric": "dense bf16 decode step (comparator, torch SDPA)", "value": top["tok_s"],
            "unit": "tok/s (best point)", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
            "higher_is_better": True, "workload": "dense", "dtype": "bf16", "data": "synthetic",
            "config": {"workload": f"dense KV comparator: ctx {ctxs} x batch {batches}, {L} layers, "
                                   f"24q/8kv heads, torch.nn.functional.scaled_dot_product_attention, "
                                   f"one CUDA graph per step", "kv_bytes_per_token_per_layer": 4096},
            "points": points,
            "roofline": {"bound": "hbm", "achieved": top["kv_gbs"], "peak": hbm, "unit": "GB/s",
                         "frac": top["kv_gbs"] / hbm, "peak_kind": peak_kind}}
    print(json.dumps(line))


# ---------------------------------------------------------------------------- main
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--batch", type=int, default=8)
    ap.add_argument("--ctx", type=int, default=4322)
    ap.add_argument("--layers", type=int, default=28)
    ap.add_argument("--cfg", default="safe")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline sample")
    ap.add_argument("--gather", default="p2p", choices=["p2p", "nccl"],
                    help="N > 1: the head outputs gathered by the decode's merge over NVLink peer "
                         "stores (p2p) or by an NCCL all-gather per layer (nccl)")
    ap.add_argument("--no-graph", action="store_true",
                    help="launch every layer eagerly instead of replaying a CUDA graph per step")
    ap.add_argument("--workload", default="decode",
                    choices=["decode", "prefill", "encode", "sweep", "dense", "ttft"],
                    help="decode: config 1 (the default line); sweep: config 2; prefill: config 3; "
                         "encode: config 4; dense: the bf16-KV comparator of configs 1 and 2; "
                         "ttft: a first chunk through the plugin (fit + write + attention)")
    ap.add_argument("--sweep-ctx", default="1082,4322,8642,14402", help="sweep: cached tokens")
    ap.add_argument("--sweep-batch", default="1,8,32,64", help="sweep: batch sizes")
    ap.add_argument("--prompt-len", type=int, default=None,
                    help="prefill: prompt tokens (7379); encode: tokens per request (16384)")
    ap.add_argument("--chunk", type=int, default=256, help="prefill: query tokens per chunk")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.workload == "dense":
        if args.steps == 200:
            args.steps = 20
        run_dense(args)
        return
    if args.workload == "sweep":
        if args.cfg == "safe" and "--cfg" not in sys.argv:
            args.cfg = "campaign4x"                 # config 2 is quoted at 4-bit storage
        if args.steps == 200:
            args.steps = 20
        run_sweep(args)
        return
    if args.workload != "decode":
        if args.prompt_len is None:
            args.prompt_len = 7379 if args.workload == "prefill" else 16384
        if args.steps == 200:                      # the decode default; these steps take seconds
            args.steps = 3
        {"prefill": run_prefill, "encode": run_encode, "ttft": run_ttft}[args.workload](args)
        return
    if args.impl == "reference":
        run_reference(args)
        return

    import torch
    import torch.distributed as dist

    from vllm_ttkv import synthetic as S
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", device_id=device, timeout=datetime.timedelta(seconds=120))
    from vllm_ttkv.shard import HeadShard
    H = 8
    sh = HeadShard(H, 24, world, rank) if world > 1 else None    # raises unless N divides the heads
    head_lo, head_hi = (sh.head_lo, sh.head_hi) if sh else (0, H)

    r1s = (S.LLAMA32_3B_R1 * ((args.layers + 27) // 28))[:args.layers]
    dense = None
    if world == 1:
        # the same step over a dense bf16 KV cache (what stock vLLM stores), torch SDPA: context for
        # the TT-KV step's time, not a measurement of this library (first, on a quiet device)
        gen = torch.Generator(device=device)
        gen.manual_seed(1)
        dense = dense_point(args.batch, args.ctx, len(r1s), min(args.steps, 50), args.warmup, device, gen)
        dense = {"ms_per_step": dense["ms_per_step"], "tok_s": dense["tok_s"], "kv_gbs": dense["kv_gbs"],
                 "api": "torch scaled_dot_product_attention over bf16 K/V, 4096 B per token per layer, "
                        "one CUDA graph per step (bench.py --workload dense sweeps it)"}
    t0 = time.perf_counter()
    wl = Workload(args.batch, args.ctx, r1s, args.cfg, device, torch.bfloat16, seed=0)
    if sh is not None:
        wl.shard(head_lo, head_hi)                 # each rank stores only its heads' rows
    setup_s = time.perf_counter() - t0

    pg = None
    gather_note = None
    if sh is not None and args.gather == "p2p":
        # the layer outputs live in memory every rank maps (CUDA IPC); the decode's merge stores
        # each row into every rank's copy and the step waits on the device for the others' rows.
        # Every rank must agree that its mappings worked; if any failed, all take the NCCL path
        from vllm_ttkv.shard import PeerGather
        err = None
        try:
            pg = PeerGather(sh, wl.L, wl.B, 128, wl.dtype, device)
        except Exception as e:                              # noqa: BLE001 (reported in the line)
            err = f"{type(e).__name__}: {e}"
        ok = torch.tensor([0 if err else 1], device=device)
        dist.all_reduce(ok, op=dist.ReduceOp.MIN)
        if int(ok.item()) == 1:
            wl.outbuf = pg.all_out.reshape(-1)
            wl.out = [pg.out(l) for l in range(wl.L)]
            wl.peers = [pg.peers(l) for l in range(wl.L)]
        else:
            if pg is not None:
                pg.close()                                  # two group barriers inside
                pg = None
            else:
                dist.barrier()                              # the same two as the others' close()
                dist.barrier()
            gather_note = "p2p set-up failed on a rank (%s); gathered by NCCL" % (err or "another rank")
            print(f"rank {rank}: {gather_note}", file=sys.stderr)
    bufs = [sh.buffers(wl.B, 128, wl.dtype, device) for _ in range(wl.L)] if sh else None

    def layer_work(l):
        """The layer's launches on this rank: write, read, and either the wait for the other
        ranks' rows (p2p) or the copy of this rank's query heads into the all-gather's send buffer."""
        wl.layer_step(l)
        if pg is not None:
            pg.wait(l)
        elif sh is not None:
            sh.pack(wl.out[l], bufs[l][0])

    graphs = None

    def step_work():
        for l in range(wl.L):
            layer_work(l)
            if sh is not None and pg is None:              # this layer's heads from every rank
                sh.gather(*bufs[l])
                sh.assemble(bufs[l][1], wl.out[l])         # every rank ends with all heads

    def run_steps(k):
        for _ in range(k):
            if graphs is not None:
                graphs[0].replay()                         # the whole step (all-gathers included)
            else:
                step_work()

    run_steps(args.warmup)
    gather_check = None
    if pg is not None:
        # once, outside the timing: every rank's gathered outputs against an NCCL all-gather of
        # the ranks' own heads (the same collectives on every rank, in the same order)
        torch.cuda.synchronize(device)
        err = 0.0
        for l in range(wl.L):
            send, recv = bufs[l]
            sh.pack(wl.out[l], send)
            sh.gather(send, recv)
            ref = torch.empty_like(wl.out[l])
            sh.assemble(recv, ref)
            err = max(err, float((ref.float() - wl.out[l].float()).abs().max().item()))
        gather_check = {"max_abs_diff_vs_nccl_all_gather": err, "layers": wl.L}
    if not args.no_graph:
        # one CUDA graph for the whole step, captured after the warm-up allocated every workspace
        # (and, on several GPUs, after the NCCL communicator ran its first collectives); the 28
        # all-gathers are captured in it. The replays launch exactly the eager steps' kernels
        torch.cuda.synchronize(device)
        graphs = [torch.cuda.CUDAGraph()]
        with torch.cuda.graph(graphs[0]):
            step_work()
        torch.cuda.synchronize(device)
    run_steps(args.warmup)
    torch.cuda.synchronize(device)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(device)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(device.index if world == 1 else local) as clk:
        torch.cuda.cudart().cudaProfilerStart()          # a profiler run with
        ev0.record()                                     # --profile-from-start off sees only
        run_steps(args.steps)                            # the timed steps
        ev1.record()
        torch.cuda.synchronize(device)
        torch.cuda.cudart().cudaProfilerStop()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(device)
    ms = ev0.elapsed_time(ev1) / args.steps
    ms_t = torch.tensor([ms], device=device)
    if world > 1:
        dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
    ms = float(ms_t.item())
    clocks = clk.summary()

    # ---- the decode launch alone, per layer, CUDA events on the launching stream
    from vllm_ttkv import ops
    n_heads = head_hi - head_lo
    reps = 3
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(wl.L * reps)]
    torch.cuda.synchronize(device)
    for rep in range(reps):
        # a few ms of device sleep first, so that the host has queued every launch of the rep
        # before the device reaches them: the events then time the device, not the host's
        # launch overhead (which exceeds a short read's device time at 4 and 8 GPUs)
        torch.cuda._sleep(int(2e7))
        for l in range(wl.L):
            a, b = evs[rep * wl.L + l]
            a.record()
            wl.read(l)
            b.record()
            if pg is not None:
                pg.wait(l)                 # (after the event) keeps the arrival counts in step
    torch.cuda.synchronize(device)
    dec_ms = [a.elapsed_time(b) for a, b in evs]
    dec_total_ms = sum(dec_ms) / reps                          # all layers' decode launches, per step
    alg_bytes = sum(wl.read_bytes(l) for l in range(wl.L))
    achieved = alg_bytes / (dec_total_ms * 1e-3) / 1e9
    # algorithmic reconstruction FLOPs, (cq*cs) @ D over the heads read (the fp16 hi/lo split of
    # D doubles the tensor-core work actually issued; that is not counted)
    recon_flops = sum(wl.B * wl.max_seq * 2 * wl.r1s[l] * n_heads * 128 for l in range(wl.L))
    hbm, tc, tc_sus, peak_kind = _peaks()

    # ---- e2e: the same step through the C-ABI with host buffers copied in and out every step:
    # every layer's q, K and V of the step in one pinned buffer, every layer's output back in one
    pin_in = wl.inbuf.cpu().pin_memory()
    pin_o = torch.empty(wl.outbuf.shape, dtype=wl.outbuf.dtype).pin_memory()
    h2d = pin_in.numel() * pin_in.element_size()
    d2h = pin_o.numel() * pin_o.element_size()

    def e2e_step():
        wl.inbuf.copy_(pin_in, non_blocking=True)
        run_steps(1)
        pin_o.copy_(wl.outbuf, non_blocking=True)

    for _ in range(2):
        e2e_step()
    torch.cuda.synchronize(device)
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        e2e_step()
    e1.record()
    torch.cuda.synchronize(device)
    e2e_ms = torch.tensor([e0.elapsed_time(e1) / args.steps], device=device)
    if world > 1:
        dist.all_reduce(e2e_ms, op=dist.ReduceOp.MAX)
    e2e_ms = float(e2e_ms.item())

    plugin = None
    if world == 1:
        p_ms, p_h2d, p_d2h = plugin_e2e(wl, args.steps, args.warmup, device)
        plugin = {"value": args.batch / (p_ms * 1e-3), "unit": "tok/s", "ms_per_step": p_ms,
                  "h2d_bytes_per_step": p_h2d, "d2h_bytes_per_step": p_d2h,
                  "api": "TTKVAttentionImpl.forward per layer (write + decode), new metadata per step"}
        g_ms, _, _ = plugin_e2e(wl, args.steps, args.warmup, device, graph=True)
        plugin["graph"] = {"value": args.batch / (g_ms * 1e-3), "unit": "tok/s", "ms_per_step": g_ms,
                           "h2d_bytes_per_step": p_h2d, "d2h_bytes_per_step": p_d2h,
                           "api": "TTKVAttentionImpl.forward x 28 captured once in a CUDA graph "
                                  "(device-planned decode step), replayed per step"}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        sl = [l for l in SAMPLE_LAYERS if l < len(r1s)]
        per = cpu_sample((args.batch, args.ctx, r1s, args.cfg), sample_layers=tuple(sl))
        cpu_step = per * args.batch * len(r1s)
        cpu = {"value": args.batch / cpu_step, "unit": "tok/s", "cores": os.cpu_count(),
               "kind": "port",
               "sample": f"{len(sl)} (request, layer) pairs (layers {sl}, r1 {[r1s[l] for l in sl]}, "
                         f"n={args.ctx}): oracle frozen write of one token + decode read, mean scaled "
                         f"x{args.batch * len(r1s)}"}

    # per layer: write (write_frozen_kernel) + read (decode kernel + merge_sk_kernel)
    launches = wl.L * (4 if pg is not None else 3)     # + the device wait of the fused gather
    cap = CAPTURED_LAUNCH["layer"]
    traffic, traffic_src = None, "no ncu capture of this kernel build"
    if CAPTURED_LAUNCH["dram_bytes"] and CAPTURED_LAUNCH["src_sha16"] == read_src_sha16() and cap < wl.L \
            and n_heads == H:
        traffic = CAPTURED_LAUNCH["dram_bytes"] * (alg_bytes / wl.L) / wl.read_bytes(cap)
        traffic_src = ("ncu dram__bytes_read+write of the layer-%d launch of %s (read sources %s), scaled "
                       "per launch by algorithmic bytes" % (cap, CAPTURED_LAUNCH["kernel"],
                                                           CAPTURED_LAUNCH["src_sha16"]))
    elif CAPTURED_LAUNCH["dram_bytes"]:
        traffic_src = "stale: the read kernel's sources changed since the ncu capture"
    if rank == 0:
        line = {"metric": METRIC, "value": args.batch / (ms * 1e-3), "unit": "tok/s",
                "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
                "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
                "dtype": "bf16 model tensors, fp32 math, u8 slots", "data": "synthetic",
                "config": {"workload": f"cfg1 decode step: B={args.batch} x {args.ctx} ctx, "
                                       f"{len(r1s)} Llama-3.2-3B layers (calibrated r1), {args.cfg}, "
                                       f"block 16",
                           "batch": args.batch, "ctx": args.ctx, "layers": len(r1s),
                           "kv_heads_per_rank": n_heads,
                           "l2": "inputs larger than L2 (slots %.0f MB/step)" % (
                               sum(wl.slot_bytes(l) for l in range(wl.L)) / 1e6),
                           "parallelism": f"kv-head shard x{world}" if world > 1 else "single",
                           "storage_bytes_per_token": sum(wl.read_layouts[l].compressed_bytes_per_token()
                                                          for l in range(wl.L)),
                           "storage": ("storage-sharded: coefficient block + this rank's heads' rows"
                                       if world > 1 else "full blobs"),
                           "launch": ("eager" if not graphs else "one CUDA graph per step" if sh is None
                                      else "one CUDA graph per step, the 28 all-gathers captured in it"
                                      if pg is None else "one CUDA graph per step, no collective in it"),
                           "gather": (None if sh is None else (gather_note or "nccl all_gather_into_tensor "
                                      "per layer") if pg is None else "fused into the decode's merge: NVLink "
                                      "peer stores into every rank's output + a device wait on signal words "
                                      "(CUDA IPC memory, no multicast)"),
                           "gather_check": gather_check},
                "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s",
                             "frac": achieved / hbm, "traffic": traffic, "peak_kind": peak_kind,
                             "kernel": "decode_tc_kernel<3> + merge_sk_kernel (ttkv_decode_paged)",
                             "alg_bytes_per_launch": alg_bytes / wl.L,
                             "launch_us": dec_total_ms * 1e3 / wl.L,
                             "traffic_source": traffic_src,
                             "tensor_tflops": recon_flops / (dec_total_ms * 1e-3) / 1e12,
                             "tensor_frac": recon_flops / (dec_total_ms * 1e-3) / 1e12 / tc_sus,
                             "tensor_peak": tc_sus, "tensor_peak_kind": "bf16 sustained (%s)" % peak_kind,
                             "decode_ms_per_step": dec_total_ms},
                "e2e": {"value": args.batch / (e2e_ms * 1e-3), "unit": "tok/s",
                        "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms},
                "gpu_launches": launches * args.steps, "clocks": clocks,
                "setup_s": round(setup_s, 1), "fit_s": round(wl.fit_s, 1)}
        if plugin is not None:
            line["e2e_plugin"] = plugin
        if dense is not None:
            line["dense_comparator"] = dense
        if cpu is not None:
            line["cpu_baseline"] = cpu
        print(json.dumps(line))
    graphs = None
    torch.cuda.synchronize(device)
    if pg is not None:
        pg.close()
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
