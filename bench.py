"""Benchmark of the compressed-KV decode path on B200.

Workload (the 32K-context decode sweep): 32 independent
layers, batch 32, 32 query / 8 KV heads, head_dim 128; per (layer, sequence, KV head)
64 cold blocks of 512 tokens at k=32 (INT8 codes + FP16 bases) and 64 hot FP16 tokens.
Caches are built by the library's own rSVD + INT8 compression from seeded
low-rank-plus-noise K/V (rank 48, sigma_i = 0.9^i, N(0, 0.05^2) noise).  One step =
one decode token for every sequence through all 32 layers (one spx_decode_attn call
over all layers), with a fresh seeded query per step.  The 26 GB of cache read per
step exceeds the 126 MB L2, so no flush is needed between steps.

Reported: decode tokens/s (value: inputs resident; e2e: through the C ABI with the
queries copied from pinned host memory and the outputs copied back every step), the
roofline of the decode launch against measured HBM bandwidth, a parity block (sampled
(layer, sequence, KV head) units of the timed configuration checked against the CPU
oracle, cos >= 0.9999 and max-abs <= 1e-2, the run exits non-zero otherwise), the
config-3 sweep of rSVD + INT8 compression (Nb 8/128/4096 x k 16/32 x 0/2 power
iterations: blocks/s, reconstruction error before and after INT8, roofline; the
4096-block k=32 q=2 point is the "rsvd" headline), config 1 on one GPU (one layer,
batch 16, 8K context: decode plus one block compression per sequence and KV head every
step, tokens/s), and the reference's own CPU code (installed under baseline/_ref) timed
on a bounded sample as the CPU baseline.

Reference arm (--impl reference): the reference package's own PyTorch CPU functions,
`kernels.spectral_attention_decode` (one (sequence, layer) decode of the workload per
step, extrapolated to a full step) and `rsvd.batched_randomized_svd`, on all host cores.

Multi-GPU (torchrun): KV heads are sharded across ranks (unsloth_spectral.sharding);
each rank decodes its head slice of every layer and one NCCL all-gather per step
assembles the outputs.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

REPO = os.path.dirname(os.path.abspath(__file__))
PKG_ROOT = os.path.join(REPO, "unsloth-spectral_b200")
REF_ROOT = os.path.join(REPO, "baseline", "_ref")
os.environ.setdefault("UNSLOTH_SPECTRAL_QUIET", "1")

import numpy as np  # noqa: E402
import torch  # noqa: E402

CFG = dict(layers=32, batch=32, q_heads=32, kv_heads=8, head_dim=128, block=512, blocks=64, rank=32, hot=64,
           gen_rank=48, rho=0.9, oversampling=8, n_iter=2, theta=1e6)
METRIC = "spectral decode-attn tokens/s & HBM GB/s at 32K ctx; rSVD blocks/s"
UNIT = "tokens/s"
WORKLOAD = "config2: 32 layers x B32 x 32/8 heads x 32K ctx (64x512 blocks, k=32) + 64 hot"
PARITY_COS, PARITY_MAXABS = 0.9999, 1e-2


def _use_ours():
    if PKG_ROOT not in sys.path:
        sys.path.insert(0, PKG_ROOT)


def algorithmic_bytes_per_step(c, kv_heads_local):
    """Bytes one decode step must move: per (layer, sequence, KV head) every cold
    block's INT8 codes (K and V), FP16 bases and scales, the FP16 hot K/V, and the
    query/output rows of its query heads."""
    nrep = c["q_heads"] // c["kv_heads"]
    per_block = c["block"] * c["rank"] * 2 + 2 * c["rank"] * c["head_dim"] * 2 + 2 * 4
    per_head = c["blocks"] * per_block + c["hot"] * c["head_dim"] * 2 * 2 + nrep * c["head_dim"] * 2 * 2
    return per_head * c["layers"] * c["batch"] * kv_heads_local


def measured_traffic(c, world):
    """DRAM bytes per decode launch from the committed ncu launch-list summary
    (profiles/decode_traffic.json), when it was taken on this exact workload."""
    p = os.path.join(REPO, "profiles", "decode_traffic.json")
    try:
        d = json.load(open(p))
    except (OSError, ValueError):
        return None, None
    if d.get("workload") != WORKLOAD or world != 1 or c["layers"] != CFG["layers"]:
        return None, None
    return d.get("dram_bytes_per_launch"), d.get("command")


def read_peaks():
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), float(d.get("bf16_tflops", 1590.0)), "measured"
    return 6650.0, 1590.0, "fallback"


def cpu_model():
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


class ClockSampler:
    """nvidia-smi samples (every 50 ms) from the warm-up through the timed region."""

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.lines = []

    def __enter__(self):
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={q}",
                                          "--format=csv,noheader,nounits", "-lms", "50"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except FileNotFoundError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# =============================================================================
# Reference arm: the reference package's own CPU code (baseline/_ref)
# =============================================================================
_REF_MODS = {}


def _import_reference():
    """Import the unmodified reference package from baseline/_ref (its own import name,
    so this process must not have imported this repository's package)."""
    if _REF_MODS:
        return _REF_MODS
    if "unsloth_spectral" in sys.modules:
        raise RuntimeError("the reference arm must run in a process without this repository's package")
    if not os.path.isdir(os.path.join(REF_ROOT, "unsloth_spectral")):
        return None
    sys.path.insert(0, REF_ROOT)
    import importlib
    import logging
    logging.disable(logging.CRITICAL)
    _REF_MODS.update({n: importlib.import_module(f"unsloth_spectral.{n}")
                      for n in ("spectral_cache", "rsvd", "kernels.spectral_attention")})
    return _REF_MODS


def _reference_cache(sc, c, seed):
    """A float32 CPU SpectralCache of one (sequence, layer) of the workload: 64 cold
    blocks of 512 tokens at k=32 (INT8-valued coefficients times a per-head scale, as
    the reference stores them) and 64 hot tokens, for 8 KV heads of D=128."""
    g = torch.Generator().manual_seed(seed)
    H, D, T, NB, R, hot = c["kv_heads"], c["head_dim"], c["block"], c["blocks"], c["rank"], c["hot"]
    cache = sc.SpectralCache(num_heads=H, head_dim=D, block_size=T, k_rank_keys=R, k_rank_values=R,
                             device="cpu", dtype=torch.float32)
    blocks = []
    for j in range(NB):
        parts = []
        for _ in range(2):
            codes = torch.randint(-127, 128, (H, T, R), generator=g).float()
            s = torch.rand(H, generator=g) * 0.01 + 0.01
            coeffs = codes * s[:, None, None]
            mm = torch.stack([coeffs.amin(dim=(1, 2)), coeffs.amax(dim=(1, 2))], dim=1)
            basis = torch.linalg.qr(torch.randn(H, D, R, generator=g))[0].transpose(1, 2).contiguous()
            parts.append((coeffs, basis, mm))
        (ck, bk, mk), (cv, bv, mv) = parts
        blocks.append(sc.SpectralBlock(coeffs_K=ck, basis_K=bk, coeffs_V=cv, basis_V=bv, scales_K=mk, scales_V=mv,
                                       block_size=T, start_position=j * T))
    cache.cold_blocks = blocks
    cache.hot_K = torch.randn(1, H, hot, D, generator=g)
    cache.hot_V = torch.randn(1, H, hot, D, generator=g)
    cache.hot_position_ids = torch.arange(NB * T, NB * T + hot).unsqueeze(0)
    cache.total_tokens = NB * T + hot
    cache.current_position = NB * T + hot
    return cache


def _rope_tables(n, D, theta):
    inv = theta ** (-2.0 * torch.arange(0, D, 2, dtype=torch.float64) / D)
    fr = torch.outer(torch.arange(n, dtype=torch.float64), inv)
    emb = torch.cat([fr, fr], dim=-1)
    return emb.cos().float(), emb.sin().float()


def reference_decode_sampler(c, seed=0):
    """Returns (call, threads, kind): ``call()`` runs one (sequence, layer) decode of the
    workload on the host cores through the reference's own
    kernels.spectral_attention_decode (kernels/spectral_attention.py:684), or through
    the numpy oracle port when the reference is not installed."""
    ncores = len(os.sched_getaffinity(0))
    torch.set_num_threads(ncores)
    mods = _import_reference()
    D, Hq = c["head_dim"], c["q_heads"]
    qpos = c["blocks"] * c["block"] + c["hot"]
    cos, sin = _rope_tables(qpos + 8, D, c["theta"])
    g = torch.Generator().manual_seed(seed + 1)
    Q = torch.randn(1, Hq, 1, D, generator=g) / math.sqrt(D)
    if mods is not None:
        ka = mods["kernels.spectral_attention"]
        cache = _reference_cache(mods["spectral_cache"], c, seed)
        cfg = ka.TritonSpectralConfig(enable_logging=False)

        def call():
            return ka.spectral_attention_decode(Q, cache, cos, sin, qpos, scale=1.0 / math.sqrt(D), config=cfg)
        return call, ncores, "reference"
    sys.path.insert(0, REPO)
    from oracle import spectral_oracle as so
    rng = np.random.default_rng(seed)
    H, T, NB, R, hot = c["kv_heads"], c["block"], c["blocks"], c["rank"], c["hot"]
    basis = np.linalg.qr(rng.standard_normal((H, D, R)))[0].transpose(0, 2, 1).astype(np.float32)
    blocks = [so.Block(rng.integers(-127, 128, size=(H, T, R)).astype(np.float32) * np.float32(0.01), basis,
                       rng.integers(-127, 128, size=(H, T, R)).astype(np.float32) * np.float32(0.01), basis, j * T)
              for j in range(NB)]
    hk = rng.standard_normal((1, H, hot, D)).astype(np.float32)
    hv = rng.standard_normal((1, H, hot, D)).astype(np.float32)
    hp = np.arange(NB * T, NB * T + hot)
    Qn, cn, sn = Q.numpy(), cos.numpy(), sin.numpy()

    def call():
        return so.spectral_attention_decode(Qn, blocks, hk, hv, hp, cn, sn, qpos)
    return call, ncores, "port"


def reference_rsvd_sample(c, nblocks=64, seed=3):
    """Time the reference's batched_randomized_svd (rsvd.py:28) on ``nblocks`` config-3
    blocks (512 x 128, rank-48 generator, k=32, q=2, p=8) on the host cores; returns
    (blocks/s, mean relative reconstruction error, threads) or None without the
    reference."""
    mods = _import_reference()
    if mods is None:
        return None
    rs = mods["rsvd"]
    torch.set_num_threads(len(os.sched_getaffinity(0)))
    g = torch.Generator().manual_seed(seed)
    M = (torch.randn(nblocks, 512, 48, generator=g) * (0.9 ** torch.arange(48))) @ torch.randn(nblocks, 48, 128,
                                                                                              generator=g)
    M = (M + 0.05 * torch.randn(nblocks, 512, 128, generator=g)).half().float()
    rs.batched_randomized_svd(M[:8], 32, n_iter=2, oversampling=8)   # warm
    t0 = time.perf_counter()
    U, S, Vh = rs.batched_randomized_svd(M, 32, n_iter=2, oversampling=8)
    dt = time.perf_counter() - t0
    err = (torch.linalg.norm(M - (U * S[:, None, :]) @ Vh, dim=(1, 2)) / torch.linalg.norm(M, dim=(1, 2)))
    return nblocks / dt, float(err.mean()), len(os.sched_getaffinity(0))


def tokens_per_s_from_call(c, per_call_s):
    """One step = batch tokens, each needing `layers` (sequence, layer) decodes."""
    return c["batch"] / (per_call_s * c["batch"] * c["layers"])


def run_reference(args, c):
    if int(os.environ.get("RANK", "0")) != 0:
        return
    call, thr, kind = reference_decode_sampler(c)
    per = []
    for s in range(args.warmup + args.steps):
        t0 = time.perf_counter()
        call()
        if s >= args.warmup:
            per.append(time.perf_counter() - t0)
    mean = sum(per) / len(per)
    v = tokens_per_s_from_call(c, mean)
    what = ("the reference's kernels.spectral_attention_decode (baseline/_ref, float32 PyTorch CPU path)"
            if kind == "reference" else "the numpy restatement of the reference (reference not installed)")
    sample = (f"each step: one (sequence, layer) decode of the workload (64 blocks x 512 at k=32 + 64 hot, "
              f"32/8 heads, D=128) by {what}; tokens/s = batch / (per-call time x batch x layers)")
    rs = reference_rsvd_sample(c) if not args.no_rsvd else None
    line = {"metric": METRIC, "value": v, "unit": UNIT, "impl": "reference", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": mean * c["batch"] * c["layers"] * 1e3,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "config": {"workload": WORKLOAD},
            "cpu_baseline": {"value": v, "unit": UNIT, "cores": thr, "kind": kind, "sample": sample,
                             "cpu_model": cpu_model(), "seconds_per_call": mean},
            "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    if rs is not None:
        line["rsvd"] = {"blocks_per_s": rs[0], "mean_rel_error": rs[1], "cores": rs[2], "blocks": 64, "k": 32,
                        "n_iter": 2, "oversampling": 8,
                        "sample": "64 of config 3's 512x128 blocks through the reference's batched_randomized_svd"}
    print(json.dumps(line), flush=True)


def cpu_baseline_subprocess(steps=4, warmup=1, timeout=600):
    """Run the reference arm in a fresh process (the reference shares this repository
    package's import name) and return its JSON line."""
    cmd = [sys.executable, os.path.abspath(__file__), "--impl", "reference", "--steps", str(steps), "--warmup",
           str(warmup)]
    env = {k: v for k, v in os.environ.items() if k not in ("RANK", "WORLD_SIZE", "LOCAL_RANK")}
    try:
        r = subprocess.run(cmd, capture_output=True, text=True, timeout=timeout, env=env)
        for ln in reversed(r.stdout.strip().splitlines()):
            if ln.startswith("{"):
                return json.loads(ln)
    except (subprocess.TimeoutExpired, ValueError):
        pass
    return None


# =============================================================================
# Our arm
# =============================================================================
def build_tiers(c, rank_id, world, dev):
    """Device tiers of this rank's KV-head slice for all layers, built by the library's
    rSVD + INT8 compression of seeded synthetic K/V.  Returns (tiers dict, rsvd seconds)."""
    from unsloth_spectral import _ops, synthetic as syn
    from unsloth_spectral.sharding import head_slice
    L, B, H, D, T, NB, R, hot = (c["layers"], c["batch"], c["kv_heads"], c["head_dim"], c["block"], c["blocks"],
                                 c["rank"], c["hot"])
    h0, h1 = head_slice(H, world, rank_id)
    Hl = h1 - h0
    t = dict(
        codes_k=torch.empty(L, B, Hl, NB, T, R, dtype=torch.int8, device=dev),
        codes_v=torch.empty(L, B, Hl, NB, R * T, dtype=torch.int8, device=dev),   # value-tile layout
        scale_k=torch.empty(L, B, Hl, NB, dtype=torch.float32, device=dev),
        scale_v=torch.empty(L, B, Hl, NB, dtype=torch.float32, device=dev),
        basis_k=torch.empty(L, B, Hl, NB, R, D, dtype=torch.float16, device=dev),
        basis_v=torch.empty(L, B, Hl, NB, R, D, dtype=torch.float16, device=dev),
        hot_k=torch.empty(L, B, Hl, hot, D, dtype=torch.float16, device=dev),
        hot_v=torch.empty(L, B, Hl, hot, D, dtype=torch.float16, device=dev),
        block_pos=torch.arange(NB, dtype=torch.int64, device=dev) * T,
        hot_pos=torch.arange(NB * T, NB * T + hot, dtype=torch.int64, device=dev),
    )
    r = R + c["oversampling"]
    nm = B * Hl * NB
    rs = 0.0
    for l in range(L):
        K, V = syn.kv_layer_batched(c.get("seed_cfg", 2), l, B, H, NB * T + hot, D, c["gen_rank"], c["rho"], dev)
        for X, name in ((K, "k"), (V, "v")):
            Xl = X[:, h0:h1].contiguous()
            t[f"hot_{name}"][l].copy_(Xl[:, :, NB * T:])
            cold = Xl[:, :, :NB * T]
            g = torch.Generator(device=dev).manual_seed(10_000 + 2 * l + (name == "v"))
            omega = torch.randn(nm, D, r, generator=g, device=dev)
            cs = (T * R, R, 1) if name == "k" else (R * T, 0, 0)
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            _ops.rsvd(cold, omega, R, c["n_iter"], want_factors=False, codes=t[f"codes_{name}"][l], codes_strides=cs,
                      rank_pad=R, qscale=t[f"scale_{name}"][l], scale_stride=1, basis=t[f"basis_{name}"][l],
                      basis_stride=R * D, M_mat_stride=T * D, num_mats=nm, m=T, n=D, codes_tiled=(name == "v"))
            torch.cuda.synchronize()
            rs += time.perf_counter() - t0
            del Xl, cold, omega
        del K, V
    return t, rs


def make_queries(c, steps, rank_id, world, cos, sin):
    """[steps][L, B, Hq_local, D] fp16 RoPE'd queries (CPU, float32 generation)."""
    from unsloth_spectral import synthetic as syn
    from unsloth_spectral.sharding import head_slice
    L, B, Hq, D = c["layers"], c["batch"], c["q_heads"], c["head_dim"]
    nrep = Hq // c["kv_heads"]
    h0, h1 = head_slice(c["kv_heads"], world, rank_id)
    qpos = c["blocks"] * c["block"] + c["hot"]
    out = []
    for s in range(steps):
        qs = []
        for l in range(L):
            q = syn.query(2, s * L + l, B, Hq, D)[:, :, 0]
            q = syn.rope_rotate(q, cos[qpos].cpu(), sin[qpos].cpu())
            qs.append(q[:, h0 * nrep:h1 * nrep])
        out.append(torch.stack(qs).to(torch.float16))
    return out, qpos


def decode_args(c, t, q, out, cos, sin, qpos, ws, Hl, freq=None):
    from unsloth_spectral import _native as N
    nrep = c["q_heads"] // c["kv_heads"]
    return N.DecodeArgs(
        num_layers=c["layers"], batch=c["batch"], num_q_heads=Hl * nrep, num_kv_heads=Hl, head_dim=c["head_dim"],
        block_size=c["block"], num_blocks=c["blocks"], block_capacity=c["blocks"], rank_k=c["rank"],
        rank_v=c["rank"], hot_len=c["hot"], hot_capacity=c["hot"], dtype=N.SPX_F16,
        rope_mode=N.SPX_ROPE_ABSOLUTE, rope_tied=1, rope_len=cos.shape[0], query_position=qpos,
        scale=1.0 / math.sqrt(c["head_dim"]), mask_stride=0, q=q.data_ptr(), codes_k=t["codes_k"].data_ptr(),
        codes_v=t["codes_v"].data_ptr(), scale_k=t["scale_k"].data_ptr(), scale_v=t["scale_v"].data_ptr(),
        basis_k=t["basis_k"].data_ptr(), basis_v=t["basis_v"].data_ptr(), block_pos=t["block_pos"].data_ptr(),
        hot_k=t["hot_k"].data_ptr(), hot_v=t["hot_v"].data_ptr(), hot_pos=t["hot_pos"].data_ptr(),
        cos_table=cos.data_ptr(), sin_table=sin.data_ptr(), mask=None, out=out.data_ptr(),
        workspace=ws.data_ptr() if ws is not None else None, workspace_bytes=ws.numel() if ws is not None else 0,
        rope_freq=freq.data_ptr() if freq is not None else None)


def parity_units(c, Hl, G=32, extra=4, seed=11):
    """(layer, sequence, local KV head) units to check: the first, middle and last
    units, both sides of the boundaries between the cold kernel's work items (items of
    G consecutive units), the last layer, plus a few seeded random ones."""
    L, B = c["layers"], c["batch"]
    n = L * B * Hl
    idx = {0, n // 2, n - 1, min(G - 1, n - 1), min(G, n - 1), min(2 * G - 1, n - 1), (L - 1) * B * Hl}
    rng = np.random.default_rng(seed)
    idx.update(int(x) for x in rng.integers(0, n, size=extra))
    out = []
    for u in sorted(idx):
        h = u % Hl
        b = (u // Hl) % B
        l = u // (Hl * B)
        out.append((l, b, h))
    return out


def parity_check(c, t, q_dev, out_dev, cos, sin, qpos, Hl, units):
    """Compare the decode output of ``units`` with the float32 CPU oracle over the same
    compressed cache (codes * scale, FP16 bases, FP16 hot tier, FP16 queries)."""
    sys.path.insert(0, REPO)
    from oracle import spectral_oracle as so
    from unsloth_spectral import _ops
    T, R, NB, D = c["block"], c["rank"], c["blocks"], c["head_dim"]
    nrep = c["q_heads"] // c["kv_heads"]
    vidx = _ops.vtile_index(T, R, "cpu")
    cos_np, sin_np = cos.cpu().numpy(), sin.cpu().numpy()
    hp = t["hot_pos"].cpu().numpy()
    bpos = t["block_pos"].cpu().numpy()
    worst_cos, worst_abs, rows = 1.0, 0.0, []
    for (l, b, h) in units:
        ck = t["codes_k"][l, b, h].cpu().float()                          # [NB, T, R]
        sk = t["scale_k"][l, b, h].cpu()
        stored = t["codes_v"][l, b, h].cpu()                              # [NB, R*T] value-tile layout
        nat = torch.empty_like(stored)
        nat[:, vidx] = stored
        cv = nat.view(NB, R, T).transpose(1, 2).float()                   # [NB, T, R]
        sv = t["scale_v"][l, b, h].cpu()
        bk = t["basis_k"][l, b, h].cpu().float()
        bv = t["basis_v"][l, b, h].cpu().float()
        blocks = [so.Block((ck[j] * sk[j]).numpy()[None], bk[j].numpy()[None], (cv[j] * sv[j]).numpy()[None],
                           bv[j].numpy()[None], int(bpos[j])) for j in range(NB)]
        hk = t["hot_k"][l, b, h].cpu().float().numpy()[None, None]
        hv = t["hot_v"][l, b, h].cpu().float().numpy()[None, None]
        Q = q_dev[l, b, h * nrep:(h + 1) * nrep].cpu().float().numpy()[None, :, None, :]
        ref = so.spectral_attention_decode(Q, blocks, hk, hv, hp, cos_np, sin_np, qpos,
                                           scale=1.0 / math.sqrt(D)).reshape(-1)
        got = out_dev[l, b, h * nrep:(h + 1) * nrep].cpu().float().numpy().reshape(-1)
        cs = float(got @ ref / (np.linalg.norm(got) * np.linalg.norm(ref) + 1e-30))
        ma = float(np.abs(got - ref).max())
        worst_cos, worst_abs = min(worst_cos, cs), max(worst_abs, ma)
        rows.append([l, b, h, round(cs, 7), ma])
    ok = bool(worst_cos >= PARITY_COS and worst_abs <= PARITY_MAXABS)
    return {"units": len(units), "cos_min": worst_cos, "max_abs": worst_abs, "passed": ok,
            "tolerance": {"cos_min": PARITY_COS, "max_abs": PARITY_MAXABS},
            "oracle": "oracle/spectral_oracle.py spectral_attention_decode (float32 numpy)",
            "sampled": rows}


# ---------------------------------------------------------------- config 3 sweep ---
# batched rSVD + INT8 quantisation of 512 x 128 FP16 blocks, Nb in
# {8, 128, 4096}, k in {16, 32}, oversampling 8, power iterations in {0, 2}; blocks are
# rank-24 (sigma_i = 0.85^i) for k = 16 and rank-48 (0.9^i) for k = 32, plus N(0, 0.05^2).
SWEEP = [(nb, k, q) for nb in (8, 128, 4096) for k in (16, 32) for q in (0, 2)]


def rsvd_blocks(nb, k, dev, seed):
    rank, rho = (24, 0.85) if k == 16 else (48, 0.9)
    g = torch.Generator(device=dev).manual_seed(seed)
    M = (torch.randn(nb, 512, rank, generator=g, device=dev) * (rho ** torch.arange(rank, device=dev))) @ \
        torch.randn(nb, rank, 128, generator=g, device=dev)
    return (M + 0.05 * torch.randn(nb, 512, 128, generator=g, device=dev)).half()


def rsvd_roofline(nb, k, q, ms, peaks):
    """Roofline of one compression call: algorithmic bytes (M read, sketch read, INT8
    codes + FP16 basis + scale written) against measured HBM bandwidth, and the
    products' FLOPs (2 + 2q products of 512 x 128 x r) against the measured bf16 peak."""
    r = k + 8
    byts = nb * (512 * 128 * 2 + 128 * r * 4 + 512 * k + k * 128 * 2 + 4)
    flops = nb * 2.0 * 512 * 128 * r * (2 + 2 * q)
    hbm, tflops = peaks
    t_hbm, t_tc = byts / (hbm * 1e9), flops / (tflops * 1e12)
    achieved = byts / (ms / 1e3) / 1e9
    return {"bound": "hbm" if t_hbm >= t_tc else "tensor", "achieved": achieved, "peak": hbm, "unit": "GB/s",
            "frac": achieved / hbm, "algorithmic_bytes": byts, "product_flops": flops,
            "tensor_frac": flops / (ms / 1e3) / (tflops * 1e12), "floor_ms": max(t_hbm, t_tc) * 1e3}


def rsvd_sweep(dev, world, stream, barrier, peaks):
    """Config 3 through spx_rsvd_compress with the cache's outputs (token-major INT8
    codes, scale, FP16 basis).  Each rank compresses nb / world blocks; time = max over
    ranks.  Errors: the rSVD's relative Frobenius reconstruction error (U S Vh) and the
    error after INT8 quantisation (codes x scale x basis), means over the blocks."""
    from unsloth_spectral import _ops
    rows = []
    for nb, k, q in SWEEP:
        nbl = nb // world
        M = rsvd_blocks(nbl, k, dev, 1000 + nb + k + q + 7 * int(os.environ.get("RANK", "0")))
        om = torch.randn(nbl, 128, k + 8, generator=torch.Generator(device=dev).manual_seed(5 + k), device=dev)
        codes = torch.empty(nbl, 512, k, dtype=torch.int8, device=dev)
        qscale = torch.empty(nbl, dtype=torch.float32, device=dev)
        basis = torch.empty(nbl, k, 128, dtype=torch.float16, device=dev)

        def call():
            _ops.rsvd(M, om, k, q, want_factors=False, codes=codes, codes_strides=(512 * k, k, 1), rank_pad=k,
                      qscale=qscale, scale_stride=1, basis=basis, basis_stride=k * 128)

        reps = 3 if nb >= 4096 else 20
        for _ in range(2):
            call()
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            call()
        e1.record(stream)
        barrier()
        ms = torch.tensor([e0.elapsed_time(e1) / reps], dtype=torch.float64, device=dev)
        if world > 1:
            torch.distributed.all_reduce(ms, op=torch.distributed.ReduceOp.MAX)
        ms = ms.item()
        U, S, Vh = _ops.rsvd(M, om, k, q, want_factors=True)
        Mf = M.float()
        den = torch.linalg.norm(Mf, dim=(1, 2))
        err = (torch.linalg.norm(Mf - (U * S[:, None, :]) @ Vh, dim=(1, 2)) / den).mean()
        Rq = (codes.float() * qscale[:, None, None]) @ basis.float()
        errq = (torch.linalg.norm(Mf - Rq, dim=(1, 2)) / den).mean()
        errs = torch.stack([err, errq]).double()
        if world > 1:
            torch.distributed.all_reduce(errs)
            errs /= world
        rows.append({"blocks": nb, "k": k, "n_iter": q, "oversampling": 8, "ms": ms,
                     "blocks_per_s": nb / (ms / 1e3), "mean_rel_error": errs[0].item(),
                     "mean_rel_error_int8": errs[1].item(), "l2": "inputs larger than L2" if nb * 131072 > 126e6
                     else "inputs fit in L2 (repeated calls)",
                     "roofline": rsvd_roofline(nb, k, q, ms, peaks)})
        del M, om, codes, qscale, basis, U, S, Vh, Mf, Rq
    return rows


# ---------------------------------------------------------------- config 1 ---------
# one layer, batch 16, 32/8 heads, 8K context = 16 cold blocks at
# k=16 + 448 warm + 64 hot tokens (512 uncompressed), rank-24 (0.85^i) + noise K/V;
# every step decodes one token per sequence AND compresses one newly full 512-token
# block per (sequence, KV head) for K and V (256 rSVDs + INT8), as SpectralCache.append
# does when its hot tier fills (spectral_cache.py:237-241).
CFG1 = dict(layers=1, batch=16, q_heads=32, kv_heads=8, head_dim=128, block=512, blocks=16, rank=16, hot=512,
            gen_rank=24, rho=0.85, oversampling=8, n_iter=2, theta=1e6, seed_cfg=1)


def run_config1(args, dev, stream, barrier):
    """Config 1 on one GPU: tokens/s of decode + per-step block compression.  The
    compression reads the 512 uncompressed tokens of every (sequence, KV head) and writes
    a spare cold slot (keys token-major, values in the value-tile layout), so the cache
    the decode reads stays the same from step to step."""
    from unsloth_spectral import _native as N, _ops
    from unsloth_spectral import synthetic as syn
    c = CFG1
    lib = N.lib_for(dev)
    L, B, H, D, T, R = c["layers"], c["batch"], c["kv_heads"], c["head_dim"], c["block"], c["rank"]
    t, _ = build_tiers(c, 0, 1, dev)
    qpos = c["blocks"] * T + c["hot"]
    cos, sin = syn.rope_tables(qpos + 16, D, c["theta"], device=dev)
    freq = _ops.rope_freq(cos, sin)
    qs, _ = make_queries(c, 4, 0, 1, cos, sin)
    qs = [q.to(dev) for q in qs]
    out = torch.empty(L, B, c["q_heads"], D, dtype=torch.float16, device=dev)
    a0 = decode_args(c, t, qs[0], out, cos, sin, qpos, None, H, freq)
    ws = torch.empty(lib.spx_decode_workspace_size(a0), dtype=torch.uint8, device=dev)
    nm = B * H
    spare = {n: dict(codes=torch.empty(nm, T * R, dtype=torch.int8, device=dev),
                     scale=torch.empty(nm, dtype=torch.float32, device=dev),
                     basis=torch.empty(nm, R, D, dtype=torch.float16, device=dev)) for n in ("k", "v")}
    om = {n: torch.randn(nm, D, R + 8, generator=torch.Generator(device=dev).manual_seed(77 + i), device=dev)
          for i, n in enumerate(("k", "v"))}
    sh = stream.cuda_stream

    def decode(i):
        a = decode_args(c, t, qs[i % 4], out, cos, sin, qpos, ws, H, freq)
        N.check(lib, lib.spx_decode_attn(a, sh), "spx_decode_attn")

    def compress():
        for n in ("k", "v"):
            sp = spare[n]
            cs = (T * R, R, 1) if n == "k" else (R * T, 0, 0)
            _ops.rsvd(t[f"hot_{n}"][0], om[n], R, c["n_iter"], want_factors=False, codes=sp["codes"],
                      codes_strides=cs, rank_pad=R, qscale=sp["scale"], scale_stride=1, basis=sp["basis"],
                      basis_stride=R * D, M_mat_stride=c["hot"] * D, num_mats=nm, m=T, n=D, codes_tiled=(n == "v"))

    def timed(fn, n):
        for i in range(3):
            fn(i)
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for i in range(n):
            fn(i)
        e1.record(stream)
        barrier()
        return e0.elapsed_time(e1) / n

    steps = max(args.steps, 10)
    step_ms = timed(lambda i: (decode(i), compress()), steps)
    dec_ms = timed(decode, steps)
    comp_ms = timed(lambda i: compress(), steps)
    decode(0)
    torch.cuda.synchronize(dev)
    par = parity_check(c, t, qs[0], out, cos, sin, qpos, H, parity_units(c, H, G=8, extra=2))
    return {"workload": "config1: 1 layer x B16 x 32/8 heads x 8K ctx (16x512 blocks, k=16) + 512 uncompressed; "
                        "per step 1 decode token per sequence + 256 block compressions (K and V, k=16, q=2)",
            "tokens_per_s": B / (step_ms / 1e3), "ms_per_step": step_ms, "decode_ms": dec_ms,
            "compress_ms": comp_ms, "blocks_compressed_per_step": 2 * nm, "steps": steps, "parity": par}


# ---------------------------------------------------------------- config 4 ---------
def run_config4(args):
    """the end-to-end greedy loop of a random-init Mistral-7B-shaped
    model (32 layers, hidden 4096, 32/8 heads, SwiGLU 14336, vocab 32768, RoPE 1e6, BF16
    weights ~ N(0, 0.02^2)) patched with patch_unsloth_attention (k=16, 512-token blocks,
    64-token hot tier): batch 8, a 4096-token random prompt, then 512 greedy tokens through
    the patched per-layer forwards (unsloth_spectral.llama_loop).  Data parallel: every
    rank runs its own replica and batch; value = all ranks' new tokens / the slowest
    rank's time (prefill + decode), timed with CUDA events."""
    _use_ours()
    from unsloth_spectral import get_cache_stats
    from unsloth_spectral.llama_loop import MISTRAL_7B, SpectralLlama
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        torch.distributed.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=900))
    B, T, NEW = 8, 4096, args.new_tokens
    t0 = time.perf_counter()
    model = SpectralLlama(MISTRAL_7B, device=dev, dtype=torch.bfloat16, seed=1234)
    model.patch(block_size=512, k_rank_keys=16, k_rank_values=16, hot_buffer_size=64)
    g = torch.Generator(device=dev).manual_seed(99 + rank)
    prompt = torch.randint(0, MISTRAL_7B.vocab, (B, T), generator=g, device=dev)
    setup_s = time.perf_counter() - t0
    stream = torch.cuda.current_stream(dev)
    model.generate(prompt, 4)   # warm-up: the same kernels, a short tail
    torch.cuda.synchronize(dev)

    def run(graphs):
        ev = {k: torch.cuda.Event(enable_timing=True) for k in ("start", "prefill", "decode")}
        if world > 1:
            torch.distributed.barrier(device_ids=[local])
        torch.manual_seed(1000 + rank)   # the rSVD sketches: the same in both runs
        ev["start"].record(stream)
        toks = model.generate(prompt, NEW, timer=lambda name: ev[name].record(stream), cuda_graphs=graphs)
        host = toks.cpu()
        torch.cuda.synchronize(dev)
        t = torch.tensor([ev["start"].elapsed_time(ev["decode"]), ev["start"].elapsed_time(ev["prefill"]),
                          ev["prefill"].elapsed_time(ev["decode"])], dtype=torch.float64, device=dev)
        if world > 1:
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        return host, t.tolist()

    eager_host, (eager_total, _, eager_decode) = run(False)
    with ClockSampler(local) as clk:
        out_host, (total_ms, prefill_ms, decode_ms) = run(True)
    same = bool(torch.equal(eager_host, out_host))
    stats = get_cache_stats(model)
    if rank == 0:
        tokens = world * B * NEW
        line = {
            "metric": "config4 end-to-end greedy tokens/s (prefill + decode) through patch_unsloth_attention",
            "value": tokens / (total_ms / 1e3), "unit": "tokens/s", "n_gpus": world, "steps": NEW, "warmup": 1,
            "ms_per_step": decode_ms / max(NEW - 1, 1), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16 weights, activations and cache tiers; INT8 cold-tier codes",
            "data": "synthetic (random-init weights, uniform random prompt ids)",
            "config": {"workload": "config4: random-init Mistral-7B shape, batch 8, 4096-token prompt, 512 greedy "
                                   "tokens, spectral cache k=16 / 512-token blocks / 64 hot",
                       "parallelism": f"batch replicas x{world}" if world > 1 else "single GPU",
                       "global_batch": world * B, "seq_len": T + NEW},
            "prefill_ms": prefill_ms, "decode_ms": decode_ms,
            "decode_tokens_per_s": world * B * (NEW - 1) / (decode_ms / 1e3),
            "decode": "CUDA graph of the per-layer patched single-token step, replayed between block "
                      "compressions (llama_loop._decode_graphed)",
            "eager": {"tokens_per_s": tokens / (eager_total / 1e3), "decode_ms": eager_decode,
                      "same_tokens_as_graphed": same},
            "e2e": {"value": tokens / (total_ms / 1e3), "unit": "tokens/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": B * 8},
            "cache_stats": {k: v for k, v in stats.items() if k != "per_layer_stats"},
            "first_tokens": out_host[0, :8].tolist(), "setup_s": setup_s, "clocks": clk.summary(),
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.barrier(device_ids=[local])
        torch.distributed.destroy_process_group()


# ---------------------------------------------------------------- kernel legs ------
def run_prefill(args):
    """The prefill attention kernel alone, one layer of config 4's prompt (batch 8, 32/8
    heads, 4096 causal tokens over a k=16 cache of 8 blocks; --small: batch 2, 2048 tokens):
    spx_prefill_attn with the causal rule, with the equivalent additive mask, and the eager
    reconstruct-and-multiply path of the reference, timed with CUDA events."""
    _use_ours()
    from unsloth_spectral import SpectralCache, _ops, integration as I, synthetic as syn
    dev = torch.device("cuda")
    dtype = torch.bfloat16
    B, H, nrep, T = (2, 8, 4, 2048) if args.small else (8, 8, 4, 4096)
    K, V = syn.kv_layer_batched(1, 0, B, H, T, 128, 24, 0.85, dev, dtype=dtype)
    cache = SpectralCache(H, 128, block_size=512, k_rank_keys=16, k_rank_values=16, device=dev, dtype=dtype)
    cache.append(K, V, torch.arange(T, device=dev)[None])
    del K, V
    cos, sin = syn.rope_tables(T + 8, 128, 1e6, device=dev)
    g = torch.Generator(device=dev).manual_seed(1)
    q = (torch.randn(B, H * nrep, T, 128, generator=g, device=dev) / math.sqrt(128) * 4).to(dtype)
    pos = torch.arange(T, device=dev)
    mask = torch.full((T, T), float("-inf"), device=dev).triu_(1)[None, None].to(dtype)

    def timed(fn, n):
        for _ in range(max(args.warmup, 1)):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(n):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / n

    causal_ms = timed(lambda: _ops.prefill(q, cache.tiers, cos, sin, pos, causal=True), args.steps)
    mask_ms = timed(lambda: _ops.prefill(q, cache.tiers, cos, sin, pos, mask=mask), args.steps)
    eager_ms = None if args.small else timed(lambda: I._dense_attention(q, cache, cos, sin, nrep, 128, mask, dtype, None), 3)
    flops = 4.0 * B * H * nrep * 128 * T * T / 2   # causal half of QK^T and PV
    print(json.dumps({"metric": "prefill attention over the compressed cache, ms per layer", "value": causal_ms,
                      "unit": "ms", "higher_is_better": False, "dtype": "bf16 (mma.sync, f32 accumulate)",
                      "config": {"workload": f"B{B} x {H * nrep}/{H} heads x {T} causal tokens, k=16 cache"},
                      "causal_tflops": flops / (causal_ms / 1e3) / 1e12, "additive_mask_ms": mask_ms,
                      "eager_reference_path_ms": eager_ms}), flush=True)


def run_rsvd(args):
    """One spx_rsvd_compress configuration (config-3 blocks, INT8 outputs) for profiling:
    --blocks, --k, --q; SPX_RSVD_PATH selects the implementation."""
    _use_ours()
    dev = torch.device("cuda")
    from unsloth_spectral import _ops
    nb, k, q = args.blocks, args.k, args.q
    M = rsvd_blocks(nb, k, dev, 7)
    om = torch.randn(nb, 128, k + 8, generator=torch.Generator(device=dev).manual_seed(5), device=dev)
    codes = torch.empty(nb, 512, k, dtype=torch.int8, device=dev)
    qs = torch.empty(nb, dtype=torch.float32, device=dev)
    basis = torch.empty(nb, k, 128, dtype=torch.float16, device=dev)

    def call():
        _ops.rsvd(M, om, k, q, want_factors=False, codes=codes, codes_strides=(512 * k, k, 1), rank_pad=k,
                  qscale=qs, scale_stride=1, basis=basis, basis_stride=k * 128)

    for _ in range(max(args.warmup, 1)):
        call()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        call()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    print(json.dumps({"metric": "rSVD + INT8 blocks/s", "value": nb / (ms / 1e3), "unit": "blocks/s", "ms": ms,
                      "config": {"blocks": nb, "k": k, "n_iter": q,
                                 "path": os.environ.get("SPX_RSVD_PATH", "auto")}}), flush=True)


class _LayerTiers:
    """One layer's slice of the bench's 32-layer storage, with the attributes the
    package's decode path reads from a cache's device tiers (no copy)."""

    def __init__(self, c, t, l):
        self.num_heads = t["codes_k"].shape[2]
        self.head_dim, self.block_size = c["head_dim"], c["block"]
        self.num_blocks = self.block_capacity = c["blocks"]
        self.rank_k = self.rank_v = self.rank_k_pad = self.rank_v_pad = c["rank"]
        self.hot_len = self.hot_capacity = c["hot"]
        self.hot_bound = None
        self.dtype, self.device = torch.float16, t["codes_k"].device
        for name in ("codes_k", "codes_v", "scale_k", "scale_v", "basis_k", "basis_v", "hot_k", "hot_v"):
            setattr(self, name, t[name][l])
        self.block_pos, self.hot_pos = t["block_pos"], t["hot_pos"]
        self._len = torch.full((), c["hot"], dtype=torch.int32, device=self.device)

    def hot_len_device(self):
        return self._len


def run_api_leg(c, t, qs_dev, cos, sin, qpos, args, stream, barrier):
    """Decode steps through the package's public entry point, one call per layer."""
    from unsloth_spectral import SpectralCache
    from unsloth_spectral.kernels import spectral_attention_decode
    L, B, D = c["layers"], c["batch"], c["head_dim"]
    caches = []
    for l in range(L):
        sc = SpectralCache(c["kv_heads"], D, block_size=c["block"], k_rank_keys=c["rank"], k_rank_values=c["rank"],
                           device=t["codes_k"].device, dtype=torch.float16)
        sc.tiers = _LayerTiers(c, t, l)
        caches.append(sc)
    nq = len(qs_dev)

    def step(i):
        q = qs_dev[i % nq]
        for l in range(L):
            spectral_attention_decode(q[l].reshape(B, -1, 1, D), caches[l], cos, sin, qpos)

    for i in range(args.warmup):
        step(i)
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(args.steps):
        step(i)
    e1.record(stream)
    barrier()
    return e0.elapsed_time(e1) / args.steps


def run_ours(args, c):
    _use_ours()
    from unsloth_spectral import _native as N, _ops
    from unsloth_spectral import synthetic as syn
    from unsloth_spectral.sharding import HeadShardGather, head_slice
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        torch.distributed.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=600))
    if c["kv_heads"] % world:
        raise SystemExit("kv heads must divide across ranks")
    h0, h1 = head_slice(c["kv_heads"], world, rank)
    Hl = h1 - h0
    nrep = c["q_heads"] // c["kv_heads"]
    Hql = Hl * nrep
    lib = N.lib_for(dev)
    L, B, D = c["layers"], c["batch"], c["head_dim"]

    t_setup = time.perf_counter()
    tiers, rsvd_setup_s = build_tiers(c, rank, world, dev)
    qpos = c["blocks"] * c["block"] + c["hot"]
    cos, sin = syn.rope_tables(qpos + 16, D, c["theta"], device=dev)
    # RoPE frequencies of the tables (host copy, read by the library at each call); the
    # reconstruct kernel runs instead when SPX_DECODE_PATH=fast
    freq = _ops.rope_freq(cos, sin)
    nq = min(args.warmup + args.steps, 16)        # distinct seeded query sets, cycled
    qs_host, _ = make_queries(c, nq, rank, world, cos, sin)
    qs_dev = [q.to(dev) for q in qs_host]
    # two output buffers: the all-gather of step i (side stream) reads one while the
    # decode of step i + 1 writes the other
    outs = [torch.empty(L, B, Hql, D, dtype=torch.float16, device=dev) for _ in range(2)]
    out = outs[0]
    a0 = decode_args(c, tiers, qs_dev[0], out, cos, sin, qpos, None, Hl, freq)
    ws = torch.empty(lib.spx_decode_workspace_size(a0), dtype=torch.uint8, device=dev)
    path = lib.spx_decode_path(a0)
    gather = HeadShardGather(out, world) if world > 1 else None
    stream = torch.cuda.current_stream(dev)
    sh = stream.cuda_stream
    setup_s = time.perf_counter() - t_setup

    def step(i, q_dev):
        o = outs[i & 1]
        if gather is not None:
            gather.release(o)
        a = decode_args(c, tiers, q_dev, o, cos, sin, qpos, ws, Hl, freq)
        N.check(lib, lib.spx_decode_attn(a, sh), "spx_decode_attn")
        if gather is not None:
            gather.start(o)

    def barrier():
        if world > 1:
            torch.distributed.barrier(device_ids=[local])
        torch.cuda.synchronize(dev)

    # ---- device-resident timing (value)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        for i in range(args.warmup):
            step(i, qs_dev[i % nq])
        barrier()
        ev0.record(stream)
        for i in range(args.steps):
            step(i, qs_dev[(args.warmup + i) % nq])
        if gather is not None:
            gather.wait()
        ev1.record(stream)
        barrier()
    dev_ms = ev0.elapsed_time(ev1)
    # per-launch time of the decode call alone (no collective)
    ev2, ev3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    ev2.record(stream)
    for i in range(args.steps):
        a = decode_args(c, tiers, qs_dev[(args.warmup + i) % nq], out, cos, sin, qpos, ws, Hl, freq)
        N.check(lib, lib.spx_decode_attn(a, sh), "spx_decode_attn")
    ev3.record(stream)
    barrier()
    kern_ms = ev2.elapsed_time(ev3) / args.steps

    # ---- end to end through the C ABI with host buffers
    pinned_in = [q.pin_memory() for q in qs_host]
    out_host = torch.empty(L, B, world * Hql, D, dtype=torch.float16).pin_memory()
    q_dev = torch.empty_like(qs_dev[0])

    def e2e_step(i):
        q_dev.copy_(pinned_in[i % nq], non_blocking=True)
        a = decode_args(c, tiers, q_dev, out, cos, sin, qpos, ws, Hl, freq)
        N.check(lib, lib.spx_decode_attn(a, sh), "spx_decode_attn")
        if gather is not None:
            gather.start(out)
            gather.wait()
            out_host.copy_(gather.assembled(), non_blocking=True)
        else:
            out_host.copy_(out, non_blocking=True)

    # one GPU: the copies run on a copy stream and overlap the neighbouring steps' decode
    # (double-buffered query and output), as a serving loop would run them; every step
    # still copies its query in from pinned host memory and its output back out, and the
    # end event waits for the last copy
    if world == 1:
        cs = torch.cuda.Stream(device=dev)
        q2 = [q_dev, torch.empty_like(q_dev)]
        o2 = [out, torch.empty_like(out)]
        oh2 = [out_host, torch.empty_like(out_host).pin_memory()]
        ev_in = [torch.cuda.Event() for _ in range(2)]
        ev_dec = [torch.cuda.Event() for _ in range(2)]
        ev_out = [torch.cuda.Event() for _ in range(2)]

        def e2e_run(i0, n):
            with torch.cuda.stream(cs):
                q2[0].copy_(pinned_in[i0 % nq], non_blocking=True)
                ev_in[0].record(cs)
            for k in range(n):
                b = k & 1
                stream.wait_event(ev_in[b])
                if k >= 2:
                    stream.wait_event(ev_out[b])   # o2[b] copied out by step k - 2
                a = decode_args(c, tiers, q2[b], o2[b], cos, sin, qpos, ws, Hl, freq)
                N.check(lib, lib.spx_decode_attn(a, sh), "spx_decode_attn")
                ev_dec[b].record(stream)
                with torch.cuda.stream(cs):
                    if k + 1 < n:
                        if k >= 1:
                            cs.wait_event(ev_dec[b ^ 1])   # q2[b ^ 1] read by step k - 1
                        q2[b ^ 1].copy_(pinned_in[(i0 + k + 1) % nq], non_blocking=True)
                        ev_in[b ^ 1].record(cs)
                    cs.wait_event(ev_dec[b])
                    oh2[b].copy_(o2[b], non_blocking=True)
                    ev_out[b].record(cs)
            stream.wait_event(ev_out[(n - 1) & 1])
            if n >= 2:
                stream.wait_event(ev_out[n & 1])

    if world == 1:
        e2e_run(0, args.warmup)
    else:
        for i in range(args.warmup):
            e2e_step(i)
    barrier()
    ev4, ev5 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev4.record(stream)
    if world == 1:
        e2e_run(args.warmup, args.steps)
    else:
        for i in range(args.steps):
            e2e_step(args.warmup + i)
    ev5.record(stream)
    barrier()
    e2e_ms = ev4.elapsed_time(ev5)

    # ---- the drop-in API: one kernels.spectral_attention_decode call per layer, over
    #      SpectralCache objects whose tiers are the layers' slices of the same storage
    api_ms = None
    if world == 1:
        api_ms = run_api_leg(c, tiers, qs_dev, cos, sin, qpos, args, stream, barrier)

    # ---- max over ranks
    times = torch.tensor([dev_ms, kern_ms, e2e_ms], dtype=torch.float64, device=dev)
    if world > 1:
        torch.distributed.all_reduce(times, op=torch.distributed.ReduceOp.MAX)
    dev_ms, kern_ms, e2e_ms = times.tolist()

    # ---- parity of the timed configuration: one more call with query set 0, sampled
    #      units checked against the CPU oracle (every rank checks its own head slice)
    a = decode_args(c, tiers, qs_dev[0], out, cos, sin, qpos, ws, Hl, freq)
    N.check(lib, lib.spx_decode_attn(a, sh), "spx_decode_attn")
    torch.cuda.synchronize(dev)
    par = parity_check(c, tiers, qs_dev[0], out, cos, sin, qpos, Hl, parity_units(c, Hl))
    # multi-GPU: the assembled output of the gathered head slices equals the local
    # slices at their global head positions
    gather_ok = None
    if gather is not None:
        gather.start(out)
        gather.wait()
        full = gather.assembled()
        gather_ok = bool(torch.equal(full[:, :, h0 * nrep:h1 * nrep], out))
    flags = torch.tensor([0.0 if par["passed"] else 1.0, 0.0 if gather_ok in (None, True) else 1.0,
                          par["cos_min"], par["max_abs"]], dtype=torch.float64, device=dev)
    if world > 1:
        worst = flags.clone()
        worst[2] = -worst[2]
        torch.distributed.all_reduce(worst, op=torch.distributed.ReduceOp.MAX)
        flags = worst
        flags[2] = -flags[2]
    par["passed"] = bool(flags[0].item() == 0.0)
    par["cos_min"], par["max_abs"] = float(flags[2].item()), float(flags[3].item())
    if gather is not None:
        par["gather_equal"] = bool(flags[1].item() == 0.0)

    # ---- config 3 (rSVD + INT8 sweep; headline point 4096 blocks, k=32, q=2) and, on one
    #      GPU, config 1 (decode + per-step block compression)
    peak, peak_tc, peak_kind = read_peaks()
    sweep = rsvd_sweep(dev, world, stream, barrier, (peak, peak_tc))
    head = next(r for r in sweep if (r["blocks"], r["k"], r["n_iter"]) == (4096, 32, 2))
    cfg1 = run_config1(args, dev, stream, barrier) if world == 1 and not args.no_config1 else None

    if rank == 0:
        tokens = B * args.steps
        value = tokens / (dev_ms / 1e3)
        e2e = tokens / (e2e_ms / 1e3)
        bytes_launch = algorithmic_bytes_per_step(c, Hl)
        achieved = bytes_launch / (kern_ms / 1e3) / 1e9
        traffic, traffic_cmd = measured_traffic(c, world)
        cpu = None
        if world == 1 and not args.no_cpu:
            cpu = cpu_baseline_subprocess()
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": dev_ms / args.steps, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None,
            "dtype": DECODE_DTYPE[path], "data": "synthetic",
            "config": {"workload": WORKLOAD,
                       "parallelism": f"kv-head shard x{world}" if world > 1 else "single GPU",
                       "l2": "inputs larger than L2 (26 GB per step)"},
            "e2e": {"value": e2e, "unit": UNIT, "h2d_bytes_per_step": qs_host[0].numel() * 2,
                    "d2h_bytes_per_step": out_host.numel() * 2},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": traffic, "traffic_command": traffic_cmd,
                         "peak_kind": peak_kind,
                         "kernel": f"spx_decode_attn ({PATH_NAMES[path]} cold tier + hot/merge)",
                         "algorithmic_bytes_per_launch": bytes_launch, "launch_ms": kern_ms},
            "parity": par,
            "rsvd": dict(head, outputs="INT8 codes + scale + FP16 basis (the cache's compression call)"),
            "rsvd_sweep": [{k: v for k, v in r.items() if k != "roofline"} | {"frac": r["roofline"]["frac"]}
                           for r in sweep],
            "config1": cfg1,
            "cpu_baseline": None,
            "clocks": clk.summary(),
            "api": None if api_ms is None else {
                "tokens_per_s": B / (api_ms / 1e3), "ms_per_step": api_ms, "calls_per_step": L,
                "path": "kernels.spectral_attention_decode once per layer (B=32, one SpectralCache per layer), "
                        "Python argument building included"},
            "gpu_launches": DECODE_LAUNCHES * args.steps,
            "setup_s": setup_s, "rsvd_setup_s": rsvd_setup_s,
        }
        if cpu is not None:
            cb = dict(cpu["cpu_baseline"])
            line["cpu_baseline"] = cb
            if "rsvd" in cpu:
                line["rsvd"]["cpu_baseline"] = cpu["rsvd"]
        print(json.dumps(line), flush=True)
    if world > 1:
        if gather is not None:
            gather.close()
        torch.distributed.barrier(device_ids=[local])
        torch.distributed.destroy_process_group()
    if cfg1 is not None and not cfg1["parity"]["passed"]:
        raise SystemExit(f"config-1 parity failed: {cfg1['parity']['cos_min']:.6f}")
    if not par["passed"]:
        raise SystemExit(f"parity failed: cos_min={par['cos_min']:.6f} max_abs={par['max_abs']:.3e}")


# What the decode call computes in, per cold-tier kernel, and how many kernels of this
# library it launches (set-up kernel, cold tier, hot tier + merge).
PATH_NAMES = {0: "generic", 1: "reconstruct", 2: "projection"}
DECODE_DTYPE = {
    0: "int8 codes + f16 bases/hot tier; f32 arithmetic throughout",
    1: ("int8 codes + f16 bases/hot tier; cold-tier keys reconstructed by tcgen05 into an f16 accumulator, RoPE "
        "in f16x2, QK and value products on f16 mma.sync with f32 accumulate; softmax and merges f32"),
    2: ("int8 codes + f16 bases/hot tier; cold-tier projections on tcgen05 with f16 operands (f16 feature table, "
        "f16 per-block projection matrix) and an f32 accumulator, scores as f32 sums of codes x projections, "
        "value product on f16 mma.sync with f32 accumulate; softmax and merges f32"),
}
DECODE_LAUNCHES = 3


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=60)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--no-rsvd", action="store_true", help="reference arm: skip the rSVD sample")
    ap.add_argument("--no-config1", action="store_true", help="skip the config-1 decode + compression leg")
    ap.add_argument("--workload", default="config2", choices=["config2", "config4", "prefill", "rsvd"],
                    help="config2: the decode benchmark (default); config4: the end-to-end model loop; "
                         "prefill / rsvd: one kernel leg (profiling)")
    ap.add_argument("--small", action="store_true", help="prefill: the small profiling case")
    ap.add_argument("--blocks", type=int, default=4096, help="rsvd: blocks per call")
    ap.add_argument("--k", type=int, default=32, help="rsvd: rank")
    ap.add_argument("--q", type=int, default=2, help="rsvd: power iterations")
    ap.add_argument("--new-tokens", type=int, default=512, help="config4: greedy tokens per sequence")
    ap.add_argument("--layers", type=int, default=None, help="override the layer count (profiling only)")
    args = ap.parse_args()
    c = dict(CFG)
    if args.layers:
        c["layers"] = args.layers
    if args.warmup < 3 and args.impl == "ours":
        print("warning: fewer than 3 warm-up steps", file=sys.stderr)
    if args.impl == "reference":
        run_reference(args, c)
    elif args.workload == "config4":
        run_config4(args)
    elif args.workload == "prefill":
        run_prefill(args)
    elif args.workload == "rsvd":
        run_rsvd(args)
    else:
        run_ours(args, c)


if __name__ == "__main__":
    main()
