"""Cached batched decode benchmark (env-steps/s) on B200.

Workload (one step = every env appends one transition token and the model
picks its next action): Qwen3-0.6B architecture truncated to 2 layers
(hidden 1024, 16 q / 8 kv heads, head_dim 128, q/k RMSNorm, RoPE theta 1e6,
intermediate 3072), random init, bf16. 256 envs per GPU whose cached context
lengths start uniform in [64, 4096]; paged KV with 128-token pages; policy
start_cache 1024 / max_cache 8192 (grow-then-rebuild, checked every step).
Each token embeds one transition id ((obs*4 + action)*2 + reward)*2 + done
(obs in [0,63], action in [0,3], reward in {0,1}, done ~ Bernoulli(0.02)):
a single discrete modality of vocab 1024. A token whose done bit is set ends
its env's task: the context is cleared and the env's next token starts a new
one (its row restarts at position 0). A 4-way DiscreteActionValueHead (fp32
RMSNorm -> SwiGLU -> linear) takes the argmax.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Multi-GPU: one process per GPU (torchrun); each rank decodes its own 256 envs
(weak scaling, no collective on the decode path); value = all ranks' env-steps
/ max-over-ranks device time.

`value` times K steps with inputs resident in HBM; `e2e` times the same steps
through the public API — the grow-then-rebuild caller loop
(GrowRebuildDecoder: policy check every step, rows re-windowed when they
need it) — with the token ids in pinned host memory (H2D copy each step) and
the actions read back to the host (D2H copy + sync each step).
`--impl reference` times the reference algorithm's CPU restatement (the
oracle; the reference itself is pure Python and is not installed on the GPU
box) on the host cores for the same metric.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

HIDDEN, LAYERS, HEADS, KV_HEADS, HEAD_DIM, INTER = 1024, 2, 16, 8, 128, 3072
ROPE_THETA = 1e6
ENVS = 256
PAGE = 128
START_CACHE, MAX_CACHE = 1024, 8192
VOCAB = 1024
LEN_LO, LEN_HI = 64, 4096


def transition_ids(rng, actions, n):
    obs = rng.integers(0, 64, size=n)
    reward = rng.integers(0, 2, size=n)
    done = (rng.random(n) < 0.02).astype(np.int64)
    return (((obs * 4 + actions) * 2 + reward) * 2 + done).astype(np.int32)


def workload_config(n_gpus):
    return {"workload": "cached batched decode, Qwen3-0.6B arch truncated to 2 layers, 256 envs/GPU, "
                        "context lengths U[64,4096], 128-token pages, start_cache 1024 / max_cache 8192, "
                        "done ~ Bernoulli(0.02) ends the env's task (context cleared, row restarts)",
            "envs_per_gpu": ENVS, "global_envs": ENVS * n_gpus, "layers": LAYERS, "hidden": HIDDEN,
            "q_heads": HEADS, "kv_heads": KV_HEADS, "head_dim": HEAD_DIM, "page_size": PAGE,
            "context_len": [LEN_LO, LEN_HI], "parallelism": f"env-sharded x{n_gpus} (no collective)",
            "l2": "inputs larger than L2: each step reads ~4.4 GB of KV per GPU"}


# ---------------------------------------------------------------- GPU arm
def build_model(seed, device):
    import torch

    from mouse_core_b200.backbone import Qwen3Backbone

    torch.manual_seed(seed)
    bb = Qwen3Backbone(hidden_dim=HIDDEN, num_layers=LAYERS, num_heads=HEADS, num_key_value_heads=KV_HEADS,
                       head_dim=HEAD_DIM, intermediate_size=INTER,
                       rope_parameters={"rope_type": "default", "rope_theta": ROPE_THETA})
    return bb.to(device=device, dtype=torch.bfloat16).eval()


class ActionHead:
    """fp32 DiscreteActionValueHead(out=4, hidden=1024, num_layers=2): RMSNorm
    (eps 1e-5) -> SwiGLU(1024 -> 1024) -> Linear(1024 -> 4) (reference
    models/heads/dqn.py:11-47, swiglu.py:13-74)."""

    def __init__(self, device, seed):
        import torch

        g = torch.Generator().manual_seed(seed)
        self.norm_w = torch.ones(HIDDEN, device=device)
        self.w1 = (torch.randn(2 * HIDDEN, HIDDEN, generator=g) / HIDDEN ** 0.5).to(device)
        self.b1 = torch.zeros(2 * HIDDEN, device=device)
        self.w2 = (torch.randn(4, HIDDEN, generator=g) / HIDDEN ** 0.5).to(device)
        self.b2 = torch.zeros(4, device=device)

    def __call__(self, h):
        import torch
        import torch.nn.functional as F

        x = F.rms_norm(h.float(), (HIDDEN,), self.norm_w, 1e-5)
        a, b = F.linear(x, self.w1, self.b1).chunk(2, dim=-1)
        return F.linear(F.silu(a) * b, self.w2, self.b2)


class Clocks:
    """SM clock and throttle-reason sampling during a timed region: an NVML
    polling thread (every ~2 ms, so short regions still get samples), or
    nvidia-smi at 200 ms when NVML is unavailable. Reads only."""

    REASONS = (("hw_slowdown", "nvmlClocksEventReasonHwSlowdown"),
               ("hw_thermal_slowdown", "nvmlClocksEventReasonHwThermalSlowdown"),
               ("sw_thermal_slowdown", "nvmlClocksEventReasonSwThermalSlowdown"),
               ("hw_power_brake_slowdown", "nvmlClocksEventReasonHwPowerBrakeSlowdown"),
               ("sw_power_cap", "nvmlClocksEventReasonSwPowerCap"))

    def __init__(self, device_index):
        import threading

        self.samples, self.reasons, self.max_mhz = [], set(), None
        self._stop = threading.Event()
        self._thread = None
        self._proc = None
        try:
            import pynvml
            import torch

            pynvml.nvmlInit()
            try:
                uuid = str(torch.cuda.get_device_properties(device_index).uuid)
                handle = pynvml.nvmlDeviceGetHandleByUUID(uuid if uuid.startswith("GPU-") else "GPU-" + uuid)
            except Exception:
                handle = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = float(pynvml.nvmlDeviceGetMaxClockInfo(handle, pynvml.NVML_CLOCK_SM))
            bits = [(name, getattr(pynvml, attr)) for name, attr in self.REASONS if hasattr(pynvml, attr)]

            def poll():
                while not self._stop.is_set():
                    try:
                        self.samples.append(float(pynvml.nvmlDeviceGetClockInfo(handle, pynvml.NVML_CLOCK_SM)))
                        active = pynvml.nvmlDeviceGetCurrentClocksEventReasons(handle)
                        for name, bit in bits:
                            if active & bit:
                                self.reasons.add(name)
                    except Exception:
                        pass
                    self._stop.wait(0.002)

            self._thread = threading.Thread(target=poll, daemon=True)
            self._thread.start()
        except Exception:
            self._start_smi(device_index)

    def _start_smi(self, device_index):
        try:
            self._proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(device_index), "--query-gpu=clocks.sm,clocks.max.sm,"
                 "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
                 "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self._proc = None

    def stop(self):
        if self._thread is not None:
            self._stop.set()
            self._thread.join(timeout=2)
        elif self._proc is not None:
            self._proc.terminate()
            try:
                out, _ = self._proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self._proc.kill()
                out, _ = self._proc.communicate()
            names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
            for line in out.strip().splitlines():
                parts = [q.strip() for q in line.split(",")]
                try:
                    self.samples.append(float(parts[0]))
                    self.max_mhz = float(parts[1])
                except (ValueError, IndexError):
                    continue
                for name, val in zip(names, parts[2:6]):
                    if val.lower() == "active":
                        self.reasons.add(name)
        else:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["clock sampling unavailable"], "samples": 0}
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None, "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


def prefill(sess, table, ctx_ids, lengths, chunk=512):
    """Feed every env's context through the session in ragged chunks."""
    import torch

    B = len(lengths)
    done = np.zeros(B, dtype=np.int64)
    while (done < lengths).any():
        n = np.minimum(lengths - done, chunk)
        S = int(n.max())
        ids = np.zeros((B, S), dtype=np.int64)
        for b in range(B):
            if n[b]:
                ids[b, S - n[b]:] = ctx_ids[b][done[b]:done[b] + n[b]]
        emb = table[torch.from_numpy(ids).to(table.device)]
        sess.forward(embeds=emb, lengths=n.tolist())
        done += n


def roofline_traffic_per_launch(algorithmic_bytes, capture="decode_attention_cfg2.json"):
    """Per-launch DRAM bytes of the split decode kernel: the DRAM / algorithmic
    byte ratio of a committed ncu capture (profiles/<capture>, a smaller
    launch of the same kernel on the same kind of workload; traffic grows with
    the KV bytes read) times this run's algorithmic bytes per launch, or None."""
    path = os.path.join(ROOT, "profiles", capture)
    try:
        with open(path) as f:
            rec = json.load(f)
        ratio = rec["capture_dram_bytes_per_launch"] / rec["capture_algorithmic_bytes_per_launch"]
        return int(ratio * algorithmic_bytes)
    except (OSError, ValueError, KeyError, ZeroDivisionError):
        return None


def run_ours(args):
    import torch
    import torch.distributed as dist

    from mouse_core_b200 import _lib
    from mouse_core_b200 import kernels as K
    from mouse_core_b200.kv_policy import resolve_cache_bounds

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)

    def barrier():
        if world > 1:
            dist.barrier()

    max_cache, start_cache = resolve_cache_bounds(MAX_CACHE, START_CACHE)
    model = build_model(0, dev)
    head = ActionHead(dev, 1)
    g = torch.Generator().manual_seed(2)
    table = (torch.randn(VOCAB, HIDDEN, generator=g)).to(device=dev, dtype=torch.bfloat16)

    # Every rank draws the same synthetic envs (contexts, tokens, task ends):
    # the per-GPU work of the weak-scaling runs is then exactly the one-GPU
    # workload, and the max-over-ranks time measures the system rather than
    # the spread between independent random draws (a few percent of device
    # time per rank on this workload's task-end resets).
    rng = np.random.default_rng(1000)
    lengths = rng.integers(LEN_LO, LEN_HI + 1, size=ENVS).astype(np.int64)
    ctx_ids = [transition_ids(rng, rng.integers(0, 4, size=L), L) for L in lengths]
    sess = model.decode_session(batch_size=ENVS, capacity=max_cache, page_size=PAGE)
    prefill(sess, table, ctx_ids, lengths)
    torch.cuda.synchronize()

    K_steps, W = args.steps, args.warmup
    total = K_steps + W
    # ---------------- device-resident loop (`value`)
    # A token whose done bit is set ends its env's task: the env's context is
    # cleared after that step and its next token starts a fresh one (the row
    # is emptied, and the device step restarts it at position 0).
    actions = rng.integers(0, 4, size=ENVS)
    n_calls = total + K_steps  # warm-up + timed, host-cost pass
    ids_host = np.stack([transition_ids(rng, actions, ENVS) for _ in range(n_calls)])
    ids_dev = torch.from_numpy(ids_host).to(dev)
    task_end = (ids_host & 1).astype(bool)
    ones = [1] * ENVS

    def embed_fn(ids):
        return table[ids]

    def act_fn(h):
        return head(h).argmax(-1)

    def device_step(i, s=sess):
        # One graph per step: embedding gather, both layers, the fp32 head and
        # the argmax (PagedDecodeSession.decode_step).
        if i > 0:
            gone = np.flatnonzero(task_end[i - 1])
            if gone.size:
                s.reset_rows(gone)
        return s.decode_step(ids_dev[i], ones, embed_fn, act_fn)

    for i in range(W):
        device_step(i)
    torch.cuda.synchronize()
    # The roofline pass below replays the timed steps on a copy of this state.
    twin = sess.clone()
    barrier()
    torch.cuda.synchronize()
    clocks = Clocks(local)
    launches0 = K.launch_count[0]
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(W, total):
        device_step(i)
    e1.record()
    torch.cuda.synchronize()
    clk = clocks.stop()
    launches = K.launch_count[0] - launches0
    ms = e0.elapsed_time(e1)
    resets_timed = int(task_end[W - 1:total - 1].sum())
    # Host cost of a step: the same steps issued one at a time onto an idle
    # GPU (synchronised before each), so no wait for the device is counted.
    host_t = []
    for i in range(total, total + K_steps):
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        device_step(i)
        host_t.append(time.perf_counter() - t0)
    torch.cuda.synchronize()
    host_us = statistics.median(host_t) * 1e6
    # Roofline pass: the timed steps again, eagerly, on the copy of the cache
    # taken before them (same tokens, same task ends, so the same KV bytes per
    # launch); each attention launch is repeated (attn_reps) between CUDA
    # events on the launching stream, the repeats queued back to back, so the
    # events time the kernel alone. The KV read per launch is larger than L2.
    twin.attn_events = []
    kv_sum = 0
    ctx_mean = []
    for i in range(W, total):
        gone = task_end[i - 1]
        kv_now = int(twin._len[~gone].sum()) + ENVS  # kv_len after this step's append
        kv_sum += kv_now
        ctx_mean.append(kv_now / ENVS)
        device_step(i, twin)
    torch.cuda.synchronize()
    attn_ms = [a.elapsed_time(b) / r for a, b, r in twin.attn_events]
    del twin
    torch.cuda.empty_cache()
    barrier()

    # ---------------- end-to-end loop through the public API (`e2e`)
    # The grow-then-rebuild caller loop (GrowRebuildDecoder, per-row): every
    # step appends each env's token to its host context, checks the policy
    # (rows_needing_rebuild against max_cache, task ends), re-windows the rows
    # that need it, and decodes; token ids go host -> device from pinned
    # memory and the actions come back to the host.
    from mouse_core_b200.grow_rebuild import GrowRebuildDecoder

    cap = int(lengths.max()) + n_calls + total + 8
    history = np.zeros((ENVS, cap), dtype=np.int32)
    ends = lengths.copy()
    for b in range(ENVS):
        history[b, :lengths[b]] = ctx_ids[b]
    rows = np.arange(ENVS)
    for i in range(n_calls):  # the host contexts of what the session now holds
        if i > 0:
            ends[task_end[i - 1]] = 0
        history[rows, ends] = ids_host[i]
        ends += 1
    dec = GrowRebuildDecoder(model, ENVS, embed_fn, max_cache=max_cache, start_cache=start_cache, per_row=True)
    dec.adopt(sess, np.zeros(ENVS, dtype=np.int64), ends)
    pending = task_end[n_calls - 1].copy()
    ends[pending] = 0
    h_act = torch.empty(ENVS, dtype=torch.int64, pin_memory=True)
    act = rng.integers(0, 4, size=ENVS)

    def e2e_step():
        nonlocal act, pending
        tok = transition_ids(rng, act, ENVS)
        history[rows, ends] = tok
        ends[:] += 1
        a, _ = dec.step(history, ends, 0, rebuild=pending, head=act_fn)
        h_act.copy_(a, non_blocking=True)
        torch.cuda.current_stream().synchronize()
        act = h_act.numpy().copy()
        pending = (tok & 1).astype(bool)
        ends[pending] = 0

    for _ in range(W):
        e2e_step()
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    rebuilt0 = dec.rows_rebuilt
    f0 = torch.cuda.Event(enable_timing=True)
    f1 = torch.cuda.Event(enable_timing=True)
    f0.record()
    for _ in range(K_steps):
        e2e_step()
    f1.record()
    torch.cuda.synchronize()
    e2e_ms = f0.elapsed_time(f1)
    e2e_rebuilt = dec.rows_rebuilt - rebuilt0
    per_rank = torch.tensor([ms / K_steps, host_us, e2e_ms / K_steps], device=dev)
    if world > 1:
        gathered = [torch.zeros_like(per_rank) for _ in range(world)]
        dist.all_gather(gathered, per_rank)
    else:
        gathered = [per_rank]
    per_rank_rows = [[round(float(x), 4) for x in t.tolist()] for t in gathered]
    ms_max = max(r[0] for r in per_rank_rows) * K_steps
    e2e_max = max(r[2] for r in per_rank_rows) * K_steps
    status = _lib.device_status()

    # Algorithmic bytes of one attention launch: K+V of every cached slot of
    # every row and kv-head (2 * Hkv * hd * 2 B per token) + q/out.
    mean_kv = kv_sum / K_steps
    attn_bytes = mean_kv * 2 * KV_HEADS * HEAD_DIM * 2 + 2 * ENVS * HEADS * HEAD_DIM * 2
    attn_avg_ms = statistics.median(attn_ms) if attn_ms else float("nan")  # a host hiccup can idle one bracket
    achieved = attn_bytes / (attn_avg_ms * 1e-3) / 1e9
    peaks = {}
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peaks = json.load(f)
    except (OSError, ValueError):
        pass
    peak = float(peaks.get("hbm_gbs", 6650.0))
    peak_src = "measured" if "hbm_gbs" in peaks else "fallback"

    del dec, sess
    torch.cuda.empty_cache()
    # The attention kernels timed alone (rank 0): bursts of a few seconds,
    # compared with the burst bf16 peak, so they run before the sustained
    # workloads below bring the GPU to its power cap (each object carries the
    # clocks it saw).
    prefill_obj = packed_obj = None
    if rank == 0 and not args.no_packed:
        prefill_obj = prefill_attention_metric(dev)
        packed_obj = packed_attention_metric(dev)
        torch.cuda.empty_cache()
    barrier()
    # The packed training step on the same ranks (strong scaling of the
    # 8-row step: rows split across ranks, one gradient all-reduce per step).
    train = None
    if not args.no_train:
        train = train_measure(dev, world, rank, local, TRAIN_ROWS, max(1, min(K_steps, args.train_steps)),
                              W)
        torch.cuda.empty_cache()
    # The large-batch decode and the GRPO branch rollout on the same ranks
    # (each rank owns its slice of envs / roots; no collective).
    large_batch = grpo = None
    if not args.no_extra:
        large_batch = large_batch_measure(dev, world, rank, local, LB["envs"], max(1, min(K_steps, args.extra_steps)),
                                          W)
        torch.cuda.empty_cache()
        grpo = grpo_measure(dev, world, rank, local, GR["roots"], max(1, min(K_steps, args.extra_steps)), W)
        torch.cuda.empty_cache()

    out = None
    if rank == 0:
        value = ENVS * world * K_steps / (ms_max * 1e-3)
        out = {
            "metric": "env-steps/s in cached batched decode",
            "value": round(value, 1),
            "unit": "env-steps/s",
            "n_gpus": world,
            "steps": K_steps,
            "warmup": W,
            "ms_per_step": round(ms_max / K_steps, 4),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic (seeded transition tokens; random-init weights)",
            "config": workload_config(world),
            "e2e": {"value": round(ENVS * world * K_steps / (e2e_max * 1e-3), 1), "unit": "env-steps/s",
                    "h2d_bytes_per_step": int(ENVS * 4 * world), "d2h_bytes_per_step": int(ENVS * 8 * world),
                    "ms_per_step": round(e2e_max / K_steps, 4)},
            "roofline": {"kernel": "split_decode_kernel (K1)", "bound": "hbm", "achieved": round(achieved, 1),
                         "peak": peak, "peak_source": peak_src, "unit": "GB/s", "frac": round(achieved / peak, 4),
                         "traffic": roofline_traffic_per_launch(attn_bytes), "algorithmic_bytes_per_launch": int(attn_bytes),
                         "median_launch_ms": round(attn_avg_ms, 5), "launches_timed": len(attn_ms)},
            "gpu_launches": int(launches),
            "clocks": clk,
            "device_status": status,
            "task_ends": {"rows_reset_in_timed_steps": resets_timed,
                          "rows_rebuilt_in_e2e_steps": int(e2e_rebuilt),
                          "mean_cached_tokens_per_row": {"first_timed_step": round(ctx_mean[0], 1),
                                                         "last_timed_step": round(ctx_mean[-1], 1)},
                          "rule": "a token with its done bit set (p = 0.02) ends the env's task: the context is "
                                  "cleared and the next token starts a fresh one (the row restarts at position 0); "
                                  "the e2e loop also checks max_cache every step (rows_needing_rebuild)"},
            "per_rank": {"fields": ["device_ms_per_step", "host_us_per_step_on_idle_gpu", "e2e_ms_per_step"],
                         "ranks": per_rank_rows},
        }
    if rank == 0 and train is not None:
        out["train"] = train
    if rank == 0 and large_batch is not None:
        out["large_batch"] = large_batch
    if rank == 0 and grpo is not None:
        out["grpo"] = grpo
    if rank == 0 and prefill_obj is not None:
        out["prefill_attention"] = prefill_obj
    if rank == 0 and packed_obj is not None:
        out["packed_attention"] = packed_obj
    # The CPU baseline is timed at N = 1 only: under torchrun the other ranks'
    # processes share the host, and the per-N comparison is the driver's
    # reference arm (rank 0 alone, the other ranks exit).
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        out["cpu_baseline"] = cpu_baseline(args.cpu_seconds)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return out


# Large-batch decode (the 8-GPU slice of a 4096-env workload): Llama-3.2-1B
# architecture (16 layers, hidden 2048, 32/8 heads, hd 64, intermediate 8192,
# RoPE theta 5e5 with rope_type "default"), 512 envs per GPU with context
# lengths log-uniform in [128, 16384], 64-token pages, and 2% of envs retiring
# every step and restarting from an empty context.
LB = {"hidden": 2048, "layers": 16, "heads": 32, "kv_heads": 8, "head_dim": 64, "inter": 8192, "theta": 5e5,
      "envs": 512, "page": 64, "len": (128, 16384), "retire": 0.02}


def large_batch_config(n_gpus, envs):
    return {"workload": f"large-batch cached decode, Llama-3.2-1B arch (16 layers, hd 64), {envs} envs/GPU "
                        "(the 8-GPU slice of 4096 envs), context lengths log-uniform [128,16384], 64-token pages, "
                        "2% of envs retire and restart each step",
            "envs_per_gpu": envs, "global_envs": envs * n_gpus, "layers": LB["layers"], "hidden": LB["hidden"],
            "q_heads": LB["heads"], "kv_heads": LB["kv_heads"], "head_dim": LB["head_dim"], "page_size": LB["page"],
            "parallelism": f"env-sharded x{n_gpus} (no collective)",
            "l2": "inputs larger than L2: each step reads ~54 GB of KV per GPU"}


def _setup_ranks():
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    return dev, world, rank, local


def _teardown_ranks(world):
    import torch.distributed as dist

    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_large_batch(args):
    dev, world, rank, local = _setup_ranks()
    out = large_batch_measure(dev, world, rank, local, args.lb_envs, args.steps, args.warmup)
    _teardown_ranks(world)
    return out


def large_batch_measure(dev, world, rank, local, envs, K_steps, W):
    """Time the large-batch decode on this process group (every rank calls
    it; rank 0 gets the result line)."""
    import torch
    import torch.distributed as dist
    import torch.nn.functional as F

    from mouse_core_b200 import _lib
    from mouse_core_b200 import kernels as K
    from mouse_core_b200.backbone import LlamaBackbone

    D, hd, Hkv, Hq, P = LB["hidden"], LB["head_dim"], LB["kv_heads"], LB["heads"], LB["page"]
    torch.manual_seed(0)
    bb = LlamaBackbone(hidden_dim=D, num_layers=LB["layers"], num_heads=Hq, num_key_value_heads=Hkv,
                       intermediate_size=LB["inter"], max_position_embeddings=32768,
                       rope_parameters={"rope_type": "default", "rope_theta": LB["theta"]})
    bb = bb.to(device=dev, dtype=torch.bfloat16).eval()
    g = torch.Generator().manual_seed(2)
    table = torch.randn(VOCAB, D, generator=g).to(device=dev, dtype=torch.bfloat16)
    w1 = (torch.randn(2 * D, D, generator=g) / D ** 0.5).to(dev)
    w2 = (torch.randn(4, D, generator=g) / D ** 0.5).to(dev)

    def head(h):  # fp32 DiscreteActionValueHead (RMSNorm -> SwiGLU -> Linear)
        a, b = F.linear(F.rms_norm(h.float(), (D,), None, 1e-5), w1).chunk(2, dim=-1)
        return F.linear(F.silu(a) * b, w2)

    rng = np.random.default_rng(3000)  # the same envs on every rank, as in the decode workload
    lo, hi = LB["len"]
    lengths = np.exp(rng.uniform(np.log(lo), np.log(hi), size=envs)).astype(np.int64)
    n_step_calls = 2 * W + 3 * K_steps  # alternating device / e2e steps, then the roofline pass
    # Exactly the pages the contexts and every timed step can need (the pool
    # never grows): each row's longest possible length plus one page of slack.
    pages = int(((lengths + n_step_calls + P - 1) // P + 1).sum())
    sess = bb.decode_session(batch_size=envs, capacity=P, page_size=P, num_pages=pages)
    ctx_ids = [transition_ids(rng, rng.integers(0, 4, size=L), L) for L in lengths]
    prefill(sess, table, ctx_ids, lengths)
    torch.cuda.synchronize()
    retire = rng.random((n_step_calls, envs)) < LB["retire"]
    ids_dev = torch.from_numpy(np.stack([transition_ids(rng, rng.integers(0, 4, size=envs), envs)
                                         for _ in range(n_step_calls)])).to(dev)
    ones = [1] * envs
    call = [0]

    def embed_fn(ids):
        return table[ids]

    def act_fn(h):
        return head(h).argmax(-1)

    def device_step():
        i = call[0]
        call[0] += 1
        gone = np.flatnonzero(retire[i])
        if gone.size:
            sess.reset_rows(gone)
        return sess.decode_step(ids_dev[i], ones, embed_fn, act_fn)

    def barrier():
        if world > 1:
            dist.barrier()

    # Retirements shrink the cached contexts step after step, so the
    # device-resident and end-to-end figures alternate step by step over the
    # same stretch of the trajectory (each step timed with its own events);
    # the roofline pass of K1 launches follows.
    h_ids = torch.empty(envs, dtype=torch.int32, pin_memory=True)
    h_act = torch.empty(envs, dtype=torch.int64, pin_memory=True)
    d_ids = torch.empty(envs, dtype=torch.int32, device=dev)
    act = rng.integers(0, 4, size=envs)

    def e2e_step():  # through the public API: ids from pinned host memory, actions read back
        nonlocal act
        i = call[0]
        call[0] += 1
        gone = np.flatnonzero(retire[i])
        if gone.size:
            sess.reset_rows(gone)
        h_ids.numpy()[:] = transition_ids(rng, act, envs)
        d_ids.copy_(h_ids, non_blocking=True)
        h_act.copy_(sess.decode_step(d_ids, ones, embed_fn, act_fn), non_blocking=True)
        torch.cuda.current_stream().synchronize()
        act = h_act.numpy().copy()

    for _ in range(W):
        device_step()
        e2e_step()
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    clocks = Clocks(local)
    launches = 0
    dev_ev, e2e_ev = [], []
    for _ in range(K_steps):
        d0, d1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        n0 = K.launch_count[0]
        d0.record()
        device_step()
        d1.record()
        launches += K.launch_count[0] - n0  # the device-resident steps' own launches
        dev_ev.append((d0, d1))
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        f0.record()
        e2e_step()
        f1.record()
        e2e_ev.append((f0, f1))
    torch.cuda.synchronize()
    clk = clocks.stop()
    ms = sum(x.elapsed_time(y) for x, y in dev_ev)
    e2e_ms = sum(x.elapsed_time(y) for x, y in e2e_ev)
    sess.attn_events = []
    kv_sum = 0
    for _ in range(K_steps):
        kv_sum += int(sess._len[~retire[call[0]]].sum()) + envs  # after this step's retirements
        device_step()
    torch.cuda.synchronize()
    attn_ms = [a.elapsed_time(b) / r for a, b, r in sess.attn_events]
    sess.attn_events = None
    t = torch.tensor([ms, e2e_ms], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max, e2e_max = (float(x) for x in t.tolist())
    status = _lib.device_status()
    attn_bytes = kv_sum / K_steps * 2 * Hkv * hd * 2 + 2 * envs * Hq * hd * 2
    attn_avg_ms = statistics.median(attn_ms) if attn_ms else float("nan")  # a host hiccup can idle one bracket
    achieved = attn_bytes / (attn_avg_ms * 1e-3) / 1e9
    peaks = {}
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peaks = json.load(f)
    except (OSError, ValueError):
        pass
    peak = float(peaks.get("hbm_gbs", 6650.0))
    out = None
    if rank == 0:
        out = {"metric": "env-steps/s in large-batch cached decode", "unit": "env-steps/s",
               "value": round(envs * world * K_steps / (ms_max * 1e-3), 1), "n_gpus": world, "steps": K_steps,
               "warmup": W, "ms_per_step": round(ms_max / K_steps, 4), "higher_is_better": True, "scaling": "weak",
               "vs_baseline": None, "dtype": "bf16",
               "data": "synthetic (seeded transition tokens; random-init weights)",
               "config": large_batch_config(world, envs),
               "e2e": {"value": round(envs * world * K_steps / (e2e_max * 1e-3), 1), "unit": "env-steps/s",
                       "h2d_bytes_per_step": int(envs * 4 * world), "d2h_bytes_per_step": int(envs * 8 * world),
                       "ms_per_step": round(e2e_max / K_steps, 4)},
               "roofline": {"kernel": "split_decode_kernel (K1), hd 64", "bound": "hbm", "achieved": round(achieved, 1),
                            "peak": peak, "peak_source": "measured" if "hbm_gbs" in peaks else "fallback",
                            "unit": "GB/s", "frac": round(achieved / peak, 4),
                            "traffic": roofline_traffic_per_launch(attn_bytes, "large_batch_split_decode_64envs.json"),
                            "algorithmic_bytes_per_launch": int(attn_bytes), "median_launch_ms": round(attn_avg_ms, 5),
                            "launches_timed": len(attn_ms)},
               "kv_pool_gb": round(pages * LB["layers"] * 2 * Hkv * P * hd * 2 / 1e9, 1),
               "gpu_launches": int(launches), "clocks": clk, "device_status": status}
    return out


# GRPO branch rollout: Qwen3-0.6B architecture cut to 8 layers; per GPU 64
# roots with contexts U[1024, 8192], each forked into 16 branches at a point
# U[1, root length] (the branch shares the root's full pages; only a partial
# last page is copied), a 256-token prefill per branch, then one-token decode
# steps of every branch (the roots sit out). 128-token pages.
GR = {"layers": 8, "roots": 64, "branches": 16, "root_len": (1024, 8192), "prefill": 256, "page": 128}


def grpo_config(n_gpus, roots):
    return {"workload": f"GRPO branch rollout, Qwen3-0.6B arch cut to 8 layers, {roots} roots/GPU with contexts "
                        f"U[1024,8192], {GR['branches']} branches per root forked at U[1, root length] sharing "
                        f"the root's pages, {GR['prefill']}-token branch prefill, then branch decode; "
                        "128-token pages",
            "roots_per_gpu": roots, "branches_per_root": GR["branches"], "layers": GR["layers"],
            "hidden": HIDDEN, "q_heads": HEADS, "kv_heads": KV_HEADS, "head_dim": HEAD_DIM,
            "page_size": GR["page"], "parallelism": f"roots sharded x{n_gpus} (no collective)",
            "l2": "inputs larger than L2: each decode step reads ~90 GB of KV per GPU"}


def unique_kv_tokens(sess, rows):
    """Distinct cached tokens that ``rows`` of a paged session read: a page
    several rows share (a forked prefix) counts once, with the most tokens
    any of them reads from it."""
    P = sess.page_size
    L = sess._len[rows]
    npg = (L + P - 1) // P
    width = int(npg.max()) if len(rows) else 0
    if width == 0:
        return 0
    cols = np.arange(width)
    held = cols[None, :] < npg[:, None]
    ids = sess.pages.table[rows][:, :width][held]
    tok = np.minimum(P, L[:, None] - cols[None, :] * P)[held]
    best = np.zeros(sess.pages.num_pages, dtype=np.int64)
    np.maximum.at(best, ids, tok)
    return int(best.sum())


def run_grpo(args):
    dev, world, rank, local = _setup_ranks()
    out = grpo_measure(dev, world, rank, local, args.grpo_roots, args.steps, args.warmup)
    _teardown_ranks(world)
    return out


def grpo_measure(dev, world, rank, local, roots, K_steps, W):
    """Time the GRPO branch rollout on this process group (every rank calls
    it; rank 0 gets the result line)."""
    import torch
    import torch.distributed as dist
    import torch.nn.functional as F

    from mouse_core_b200 import _lib
    from mouse_core_b200 import kernels as K
    from mouse_core_b200.backbone import Qwen3Backbone

    def barrier():
        if world > 1:
            dist.barrier()

    R, G, P, D = roots, GR["branches"], GR["page"], HIDDEN
    NB = R * G
    B = R + NB
    torch.manual_seed(0)
    bb = Qwen3Backbone(hidden_dim=D, num_layers=GR["layers"], num_heads=HEADS, num_key_value_heads=KV_HEADS,
                       head_dim=HEAD_DIM, intermediate_size=INTER,
                       rope_parameters={"rope_type": "default", "rope_theta": ROPE_THETA})
    bb = bb.to(device=dev, dtype=torch.bfloat16).eval()
    g = torch.Generator().manual_seed(2)
    table = torch.randn(VOCAB, D, generator=g).to(device=dev, dtype=torch.bfloat16)
    head = ActionHead(dev, 1)

    rng = np.random.default_rng(5000)  # the same roots on every rank, as in the decode workload
    lo, hi = GR["root_len"]
    root_len = rng.integers(lo, hi + 1, size=R)
    fork_at = rng.integers(1, np.repeat(root_len, G) + 1)  # per branch, U[1, root length]
    n_step_calls = W + 2 * K_steps + W + K_steps
    pages = int(((root_len + P - 1) // P).sum() + ((fork_at % P) > 0).sum()
                + NB * ((GR["prefill"] + n_step_calls + 2 * P - 1) // P) + 8)
    sess = bb.decode_session(batch_size=B, capacity=P, page_size=P, num_pages=pages)
    lengths = np.concatenate([root_len, np.zeros(NB, dtype=np.int64)])
    ctx_ids = [transition_ids(rng, rng.integers(0, 4, size=int(L)), int(L)) for L in lengths]
    prefill(sess, table, ctx_ids, lengths)
    root_pages = sess.pages.num_pages - sess.pages.free_pages
    sess.fork(np.repeat(np.arange(R), G), R + np.arange(NB), fork_at)
    fork_pages = sess.pages.num_pages - sess.pages.free_pages - root_pages
    unshared_pages = int(((fork_at + P - 1) // P).sum())  # the same prefixes copied per branch
    page_bytes = GR["layers"] * 2 * KV_HEADS * P * HEAD_DIM * 2

    # Branch prefill (timed on its own): 256 tokens per branch, roots sit out.
    S = GR["prefill"]
    pre_ids = torch.from_numpy(rng.integers(0, VOCAB, size=(B, S))).to(dev)
    pre_len = [0] * R + [S] * NB
    torch.cuda.synchronize()
    p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    p0.record()
    sess.forward(embeds=table[pre_ids], lengths=pre_len)
    p1.record()
    torch.cuda.synchronize()
    prefill_ms = p0.elapsed_time(p1)

    step_len = [0] * R + [1] * NB
    ids_dev = torch.from_numpy(np.stack([transition_ids(rng, rng.integers(0, 4, size=B), B)
                                         for _ in range(n_step_calls)])).to(dev)
    call = [0]

    def embed_fn(ids):
        return table[ids]

    def act_fn(h):  # the branches' actions (the roots sit out)
        return head(h[R:]).argmax(-1)

    def device_step():
        i = call[0]
        call[0] += 1
        return sess.decode_step(ids_dev[i], step_len, embed_fn, act_fn)

    for _ in range(W):
        device_step()
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    clocks = Clocks(local)
    launches0 = K.launch_count[0]
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(K_steps):
        device_step()
    e1.record()
    torch.cuda.synchronize()
    clk = clocks.stop()
    launches = K.launch_count[0] - launches0
    ms = e0.elapsed_time(e1)
    sess.attn_events = []
    kv_sum = 0
    for _ in range(K_steps):
        # Shared prefix pages are read by every branch of a root but count once.
        kv_sum += unique_kv_tokens(sess, np.arange(R, B)) + NB
        device_step()
    torch.cuda.synchronize()
    attn_ms = [a.elapsed_time(b) / r for a, b, r in sess.attn_events]
    sess.attn_events = None

    h_ids = torch.empty(B, dtype=torch.int32, pin_memory=True)
    h_act = torch.empty(NB, dtype=torch.int64, pin_memory=True)
    d_ids = torch.empty(B, dtype=torch.int32, device=dev)
    act = rng.integers(0, 4, size=B)

    def e2e_step():  # through the public API: ids from pinned host memory, actions read back
        nonlocal act
        call[0] += 1
        h_ids.numpy()[:] = transition_ids(rng, act, B)
        d_ids.copy_(h_ids, non_blocking=True)
        h_act.copy_(sess.decode_step(d_ids, step_len, embed_fn, act_fn), non_blocking=True)
        torch.cuda.current_stream().synchronize()
        act[R:] = h_act.numpy()

    for _ in range(W):
        e2e_step()
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record()
    for _ in range(K_steps):
        e2e_step()
    f1.record()
    torch.cuda.synchronize()
    e2e_ms = f0.elapsed_time(f1)
    t = torch.tensor([ms, e2e_ms, prefill_ms], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max, e2e_max, pre_max = (float(x) for x in t.tolist())
    status = _lib.device_status()
    attn_bytes = kv_sum / K_steps * 2 * KV_HEADS * HEAD_DIM * 2 + 2 * B * HEADS * HEAD_DIM * 2
    attn_avg_ms = statistics.median(attn_ms) if attn_ms else float("nan")  # a host hiccup can idle one bracket
    achieved = attn_bytes / (attn_avg_ms * 1e-3) / 1e9
    peaks = {}
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peaks = json.load(f)
    except (OSError, ValueError):
        pass
    peak = float(peaks.get("hbm_gbs", 6650.0))
    out = None
    if rank == 0:
        out = {"metric": "branch env-steps/s in GRPO rollout decode", "unit": "env-steps/s",
               "value": round(NB * world * K_steps / (ms_max * 1e-3), 1), "n_gpus": world, "steps": K_steps,
               "warmup": W, "ms_per_step": round(ms_max / K_steps, 4), "higher_is_better": True, "scaling": "weak",
               "vs_baseline": None, "dtype": "bf16",
               "data": "synthetic (seeded transition tokens; random-init weights)",
               "config": grpo_config(world, R),
               "e2e": {"value": round(NB * world * K_steps / (e2e_max * 1e-3), 1), "unit": "env-steps/s",
                       "h2d_bytes_per_step": int(B * 4 * world), "d2h_bytes_per_step": int(NB * 8 * world),
                       "ms_per_step": round(e2e_max / K_steps, 4)},
               "branch_prefill": {"tokens_per_s": round(NB * S * world / (pre_max * 1e-3), 1),
                                  "ms": round(pre_max, 3)},
               "prefix_sharing": {"root_kv_gb": round(root_pages * page_bytes / 1e9, 2),
                                  "branch_prefix_kv_gb_if_copied": round(unshared_pages * page_bytes / 1e9, 2),
                                  "branch_prefix_kv_gb_with_sharing": round(fork_pages * page_bytes / 1e9, 2)},
               "roofline": {"kernel": "split_decode_kernel (K1)", "bound": "hbm", "achieved": round(achieved, 1),
                            "peak": peak, "peak_source": "measured" if "hbm_gbs" in peaks else "fallback",
                            "unit": "GB/s", "frac": round(achieved / peak, 4),
                            "traffic": roofline_traffic_per_launch(attn_bytes, "grpo_split_decode_8roots.json"),
                            "algorithmic_bytes_per_launch": int(attn_bytes), "median_launch_ms": round(attn_avg_ms, 5),
                            "launches_timed": len(attn_ms),
                            "note": "algorithmic bytes count each distinct cached token once per launch: a "
                                    "prefix page the 16 branches of a root share is counted once"},
               "cpu_baseline": None,
               "cpu_baseline_note": "not run: one step reads ~90 GB of KV; the decode line's CPU port covers the "
                                    "same per-token arithmetic",
               "gpu_launches": int(launches), "clocks": clk, "device_status": status}
    return out


def packed_segments(seed, rows=8, row_len=16384, lo=256, hi=4096):
    """Segment lengths of the packed-training workload: per row, lengths
    U[lo, hi] until the row is full, the last one truncated."""
    rng = np.random.default_rng(seed)
    segs = []
    for _ in range(rows):
        total = 0
        while total < row_len:
            s = min(int(rng.integers(lo, hi + 1)), row_len - total)
            segs.append(s)
            total += s
    return segs


def packed_attention_metric(device, reps=10, rows=8):
    """Forward TFLOP/s of the K5 segment-causal attention on the packed
    training workload's attention shape: 8 rows x 16384 tokens (one stream of
    131072), segments U[256,4096], 16 q / 8 kv heads, hd 128, bf16. Algorithmic
    FLOPs = 4 * Hq * hd * sum_s s(s+1)/2 (only unmasked pairs)."""
    import torch

    from mouse_core_b200 import kernels as K

    segs = packed_segments(0, rows=rows)
    seq = np.concatenate([np.full(n, i, dtype=np.int64) for i, n in enumerate(segs)])
    L, Hq, Hkv, hd = seq.shape[0], 16, 8, 128
    g = torch.Generator(device=device).manual_seed(0)
    q = torch.randn(L, Hq, hd, generator=g, device=device).bfloat16()
    k = torch.randn(L, Hkv, hd, generator=g, device=device).bfloat16()
    v = torch.randn(L, Hkv, hd, generator=g, device=device).bfloat16()
    _, rs, tl, _, re = K.segment_meta(torch.from_numpy(seq).to(device), tile=128, with_run_end=True)
    flops = 4 * Hq * hd * sum(s * (s + 1) // 2 for s in segs)
    do = torch.randn(L, Hq, hd, generator=g, device=device).bfloat16()
    scale = hd ** -0.5

    def timed(fn):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / reps

    from mouse_core_b200.packed import pair_count

    pair_off = K.varlen_pair_offsets(tl, L)
    n_pairs = pair_count(seq)
    out, lse = K.varlen_attention_fwd(q, k, v, rs, tl, scale)
    ms_recompute = timed(lambda: K.varlen_attention_bwd(q, k, v, out, do, lse, rs, re, scale))
    clocks = Clocks(device.index or 0)
    ms = timed(lambda: K.varlen_attention_fwd(q, k, v, rs, tl, scale))
    ms_bwd = timed(lambda: K.varlen_attention_bwd(q, k, v, out, do, lse, rs, re, scale, tile_lo=tl,
                                                  pair_off=pair_off, n_pairs=n_pairs))
    clk = clocks.stop()
    peaks = {}
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peaks = json.load(f)
    except (OSError, ValueError):
        pass
    peak = float(peaks.get("bf16_tflops", 1590.0))
    peak_sus = peaks.get("bf16_tflops_sustained")
    tf = flops / (ms * 1e-3) / 1e12
    tf_bwd = 2.5 * flops / (ms_bwd * 1e-3) / 1e12
    tf_rec = 2.5 * flops / (ms_recompute * 1e-3) / 1e12
    tf_all = 3.5 * flops / ((ms + ms_bwd) * 1e-3) / 1e12
    from mouse_core_b200 import _lib

    status = _lib.device_status()
    return {"device_status": status,
            "metric": "packed varlen segment-causal attention fwd+bwd TFLOP/s",
            "workload": f"{L} tokens ({rows} x 16384), {len(segs)} segments U[256,4096], 16/8 heads, hd 128, bf16",
            "value": round(tf_all, 1), "unit": "TFLOP/s", "algorithmic_flops_fwd": flops,
            "flops_note": "algorithmic = 4*Hq*hd*sum s(s+1)/2 (unmasked pairs only); bwd counted as 2.5x fwd",
            "peak_note": "frac: of the measured burst bf16 peak; frac_of_sustained: of the cuBLAS rate measured "
                         "under the same power cap a seconds-long tensor loop meets (the clocks below say which "
                         "regime this run was in)",
            "fwd": {"ms": round(ms, 4), "tflops": round(tf, 1), "frac": round(tf / peak, 4),
                    "frac_of_sustained": round(tf / float(peak_sus), 4) if peak_sus else None},
            "bwd": {"ms": round(ms_bwd, 4), "tflops": round(tf_bwd, 1), "frac": round(tf_bwd / peak, 4),
                    "frac_of_sustained": round(tf_bwd / float(peak_sus), 4) if peak_sus else None,
                    "path": f"stored dS ({n_pairs} pairs x {Hq} heads x 32 KB = {Hq * n_pairs * 32768 / 2**30:.2f} GiB)"},
            "bwd_recompute": {"ms": round(ms_recompute, 4), "tflops": round(tf_rec, 1),
                              "frac": round(tf_rec / peak, 4)},
            "clocks": clk,
            "roofline": {"bound": "tensor", "achieved": round(tf_all, 1), "peak": peak,
                         "peak_source": "measured" if "bf16_tflops" in peaks else "fallback",
                         "unit": "TFLOP/s", "frac": round(tf_all / peak, 4),
                         "frac_of_sustained": round(tf_all / float(peak_sus), 4) if peak_sus else None}}


def prefill_attention_metric(device, reps=5):
    """TFLOP/s of the tcgen05 paged prefill attention (one layer's K/V pool):
    the GRPO branch prefill shape (256 rows each prefilling 256 tokens over a
    cached context U[1024, 8192]) and the grow-then-rebuild prefill (256 rows
    each re-prefilling a 1024-token window from an empty cache). Qwen3-0.6B
    heads (16 q / 8 kv, hd 128), 128-token pages scattered through the pool.
    Algorithmic FLOPs = 4 * Hq * hd * sum over real queries of the keys each
    one sees."""
    import torch

    from mouse_core_b200 import kernels as K

    peaks = {}
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peaks = json.load(f)
    except (OSError, ValueError):
        pass
    peak = float(peaks.get("bf16_tflops", 1590.0))
    rng = np.random.default_rng(11)
    Hq, Hkv, hd, page = HEADS, KV_HEADS, HEAD_DIM, PAGE
    res = {}
    clocks = Clocks(device.index or 0)
    for name, B, S, ctx in (("branch_prefill", 256, 256, rng.integers(1024, 8193, size=256)),
                            ("rebuild_prefill", 256, 1024, np.zeros(256, dtype=np.int64))):
        lens = (ctx + S).astype(np.int64)
        npg = (lens + page - 1) // page
        P = int(npg.sum())
        perm = rng.permutation(P).astype(np.int32)
        bt = np.full((B, int(npg.max())), -1, dtype=np.int32)
        o = 0
        for b in range(B):
            bt[b, :npg[b]] = perm[o:o + npg[b]]
            o += npg[b]
        g = torch.Generator(device=device).manual_seed(3)
        kp = torch.randn(P, Hkv, page, hd, generator=g, device=device).bfloat16()
        vp = torch.randn(P, Hkv, page, hd, generator=g, device=device).bfloat16()
        q = torch.randn(B, S, Hq, hd, generator=g, device=device).bfloat16()
        q_pos = torch.from_numpy((ctx[:, None] + np.arange(S)[None, :]).astype(np.int32)).to(device)
        kv_len = torch.from_numpy(lens.astype(np.int32)).to(device)
        btd = torch.from_numpy(bt).to(device)
        out = torch.empty_like(q)
        flops = 4 * Hq * hd * int(sum(S * int(c) + S * (S + 1) // 2 for c in ctx))

        ws = torch.empty(256, dtype=torch.uint8, device=device)  # the persistent CTAs' tile counter

        def run():
            K.decode_attention(q, kp, vp, btd, q_pos, kv_len, hd ** -0.5, int(lens.max()), out=out, workspace=ws)

        for _ in range(2):
            run()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            run()
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / reps
        tf = flops / (ms * 1e-3) / 1e12
        res[name] = {"rows": B, "queries_per_row": S, "context": "U[1024,8192]" if ctx.any() else "empty",
                     "ms": round(ms, 4), "tflops": round(tf, 1), "frac": round(tf / peak, 4),
                     "algorithmic_flops": flops}
        del kp, vp, q, out
        torch.cuda.empty_cache()
    return {"kernel": "varlen_fwd_kernel<PAGED> (tcgen05 paged prefill, one layer)", "bound": "tensor",
            "peak": peak, "peak_source": "measured" if "bf16_tflops" in peaks else "fallback", "unit": "TFLOP/s",
            **res, "clocks": clocks.stop()}


# ------------------------------------------------------- packed training
TRAIN_LAYERS, TRAIN_ROWS, TRAIN_ROW_LEN = 28, 8, 16384


def train_config(n_gpus, rows=TRAIN_ROWS):
    return {"workload": f"packed DQN training step, Qwen3-0.6B arch (28 layers), {rows} rows x 16384 tokens, "
                        "segments U[256,4096] (last truncated per row), synthetic transition tokens, "
                        "Q targets U[0,1]^4 in place of the target head, AdamW",
            "rows": rows, "row_len": TRAIN_ROW_LEN, "layers": TRAIN_LAYERS, "hidden": HIDDEN, "q_heads": HEADS,
            "kv_heads": KV_HEADS, "head_dim": HEAD_DIM, "intermediate": INTER,
            "parallelism": f"dp{n_gpus} (rows split across ranks; one fp32 gradient all-reduce per step)",
            "l2": "inputs larger than L2: each layer's activations of one row are ~1 GB"}


def train_row_segments(seed=0, rows=TRAIN_ROWS, row_len=TRAIN_ROW_LEN, lo=256, hi=4096):
    """Per-row segment lengths: U[lo, hi] until the row is full, the last truncated."""
    rng = np.random.default_rng(seed)
    out = []
    for _ in range(rows):
        segs, total = [], 0
        while total < row_len:
            s = min(int(rng.integers(lo, hi + 1)), row_len - total)
            segs.append(s)
            total += s
        out.append(segs)
    return out


def train_row_host(seed, segs):
    """One packed row in host memory: transition token ids and the fields the
    TD loss reads (action, reward, done code), sequence ids, U[0,1]^4 targets."""
    rng = np.random.default_rng(seed)
    n = int(sum(segs))
    obs = rng.integers(0, 64, size=n)
    action = rng.integers(0, 4, size=n)
    reward = rng.integers(0, 2, size=n)
    done = (rng.random(n) < 0.02).astype(np.int64)
    ids = (((obs * 4 + action) * 2 + reward) * 2 + done).astype(np.int64)
    seq = np.concatenate([np.full(s, i, dtype=np.int64) for i, s in enumerate(segs)])
    return {"token_ids": ids, "sequence_ids": seq, "action": action.astype(np.int64),
            "reward": reward.astype(np.float32), "done": done, "q_target": rng.random((n, 4), dtype=np.float32)}


def train_flops(segs_per_row, n_params):
    """Algorithmic FLOPs of one training step over the given rows: 6 * params
    * tokens for the linear layers + 3.5x the segment-causal attention
    forward (4 * Hq * hd * sum s(s+1)/2 per layer)."""
    tokens = sum(sum(s) for s in segs_per_row)
    attn_fwd = 4 * HEADS * HEAD_DIM * TRAIN_LAYERS * sum(x * (x + 1) // 2 for s in segs_per_row for x in s)
    return 6 * n_params * tokens + 3.5 * attn_fwd, attn_fwd


def run_train(args):
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    out = train_measure(dev, world, rank, local, args.train_rows, args.steps, args.warmup)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return out


def train_measure(dev, world, rank, local, rows_total, K_steps, W):
    """Time the packed DQN training step on this process group (every rank
    calls it; rank 0 gets the result line, the others None)."""
    import torch
    import torch.distributed as dist

    from mouse_core_b200 import _lib
    from mouse_core_b200 import kernels as K
    from mouse_core_b200.backbone import Qwen3Backbone
    from mouse_core_b200.train import ActionValueHead, PackedDQNTrainer, PackedRow

    def barrier():
        if world > 1:
            dist.barrier()
    torch.manual_seed(0)
    bb = Qwen3Backbone(hidden_dim=HIDDEN, num_layers=TRAIN_LAYERS, num_heads=HEADS, num_key_value_heads=KV_HEADS,
                       head_dim=HEAD_DIM, intermediate_size=INTER,
                       rope_parameters={"rope_type": "default", "rope_theta": ROPE_THETA})
    bb = bb.to(device=dev, dtype=torch.bfloat16).train()
    emb = torch.nn.Embedding(VOCAB, HIDDEN).to(device=dev, dtype=torch.bfloat16)
    head = ActionValueHead(HIDDEN, 4).to(dev)
    params = list(emb.parameters()) + list(bb.model.parameters()) + list(head.parameters())
    opt = torch.optim.AdamW(params, lr=1e-5, fused=True)
    trainer = PackedDQNTrainer(emb, bb.model, head, opt)
    n_backbone = sum(p.numel() for n, p in bb.model.named_parameters() if "embed_tokens" not in n)

    segs = train_row_segments(0, rows=rows_total)
    mine = list(range(rank, rows_total, world))
    host = [train_row_host(100 + i, segs[i]) for i in mine]

    def to_dev(r, pinned=None):
        src = pinned if pinned is not None else {k: torch.from_numpy(v) for k, v in r.items()}
        return PackedRow(**{k: t.to(dev, non_blocking=True) for k, t in src.items()})

    resident = [to_dev(r) for r in host]
    pinned = [{k: torch.from_numpy(v).pin_memory() for k, v in r.items()} for r in host]
    h2d_bytes = sum(t.numel() * t.element_size() for p in pinned for t in p.values()) * world

    for _ in range(W):
        trainer.step(resident, rows_total)
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    clocks = Clocks(local)
    launches0 = K.launch_count[0]
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(K_steps):
        loss = trainer.step(resident, rows_total)
    e1.record()
    torch.cuda.synchronize()
    clk = clocks.stop()
    launches = K.launch_count[0] - launches0
    ms = e0.elapsed_time(e1)
    ms_t = torch.tensor([ms], device=dev)
    if world > 1:
        dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
    ms_max = float(ms_t.item())

    # End to end: every step copies its rows from pinned host memory and
    # reads the loss back.
    h_loss = torch.empty((), dtype=torch.float32, pin_memory=True)
    barrier()
    torch.cuda.synchronize()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record()
    for _ in range(K_steps):
        rows = [to_dev(None, p) for p in pinned]
        h_loss.copy_(trainer.step(rows, rows_total), non_blocking=True)
        torch.cuda.current_stream().synchronize()
    f1.record()
    torch.cuda.synchronize()
    et = torch.tensor([f0.elapsed_time(f1)], device=dev)
    if world > 1:
        dist.all_reduce(et, op=dist.ReduceOp.MAX)
    e2e_max = float(et.item())
    status = _lib.device_status()

    flops, attn_fwd = train_flops(segs, n_backbone)
    peaks = {}
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peaks = json.load(f)
    except (OSError, ValueError):
        pass
    peak = float(peaks.get("bf16_tflops_sustained", peaks.get("bf16_tflops", 1400.0)))
    out = None
    if rank == 0:
        tokens = rows_total * TRAIN_ROW_LEN
        achieved = flops * K_steps / (ms_max * 1e-3) / 1e12 / world  # per GPU, against one GPU's peak
        out = {"metric": "tokens/s in packed DQN training (fwd+bwd+AdamW)",
               "value": round(tokens * K_steps / (ms_max * 1e-3), 1), "unit": "tokens/s", "n_gpus": world,
               "steps": K_steps, "warmup": W, "ms_per_step": round(ms_max / K_steps, 3), "higher_is_better": True,
               "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
               "data": "synthetic (seeded transition tokens and U[0,1]^4 Q targets; random-init weights)",
               "config": train_config(world, rows_total),
               "e2e": {"value": round(tokens * K_steps / (e2e_max * 1e-3), 1), "unit": "tokens/s",
                       "h2d_bytes_per_step": int(h2d_bytes), "d2h_bytes_per_step": 4 * world,
                       "ms_per_step": round(e2e_max / K_steps, 3)},
               "roofline": {"kernel": "whole step (cuBLAS GEMMs + K5/K6 attention)", "bound": "tensor",
                            "achieved": round(achieved, 1), "peak": peak,
                            "peak_source": "measured (sustained)" if "bf16_tflops_sustained" in peaks else "fallback",
                            "unit": "TFLOP/s", "frac": round(achieved / peak, 4), "traffic": None,
                            "flops_note": "per GPU: (6 * 440.4M params * tokens + 3.5 x algorithmic attention "
                                          "forward) / n_gpus"},
               "attention_fwd_flops_per_step": attn_fwd, "loss": float(loss.item()),
               "gpu_launches": int(launches), "clocks": clk, "device_status": status,
               "all_reduce": "one logical fp32 all-reduce per step in 64 MB buckets launched from backward "
                             "hooks during the last row's backward (none with one GPU)"}
    return out


# ---------------------------------------------------------------- CPU arm
def _oracle_decoder(seed):
    """The bench model's architecture as a float64 oracle decoder (weights
    drawn from the same seed on the CPU)."""
    import torch

    from mouse_core_b200.backbone import Qwen3Backbone
    from oracle import decoder as odec

    torch.manual_seed(seed)
    bb = Qwen3Backbone(hidden_dim=HIDDEN, num_layers=LAYERS, num_heads=HEADS, num_key_value_heads=KV_HEADS,
                       head_dim=HEAD_DIM, intermediate_size=INTER,
                       rope_parameters={"rope_type": "default", "rope_theta": ROPE_THETA})
    sd = {k: v.detach().float().numpy() for k, v in bb.model.state_dict().items() if "rotary" not in k}
    cfg = odec.config_from_hf(bb.model.config, bb.model.rotary_emb.inv_freq.numpy())
    return odec.DecoderOracle(sd, cfg)


def _usable_cores():
    """Cores this process may run on: its CPU affinity, capped by a cgroup
    CPU quota when one is set (a container's share of a larger host)."""
    try:
        n = len(os.sched_getaffinity(0))
    except (AttributeError, OSError):
        n = os.cpu_count() or 1
    try:
        with open("/sys/fs/cgroup/cpu.max") as f:
            quota, period = f.read().split()[:2]
        if quota != "max" and int(period) > 0:
            n = min(n, max(1, -(-int(quota) // int(period))))
    except (OSError, ValueError):
        pass
    return max(1, n)


def _host_threads():
    """Give numpy's BLAS and torch every usable host core (torchrun sets
    OMP_NUM_THREADS=1 for its ranks) and return the thread count in use."""
    import torch
    from threadpoolctl import threadpool_info, threadpool_limits

    n = _usable_cores()
    threadpool_limits(limits=n)
    torch.set_num_threads(n)
    blas = [i.get("num_threads", 1) for i in threadpool_info() if i.get("user_api") == "blas"]
    return max(blas) if blas else torch.get_num_threads()


def cpu_baseline(seconds=15.0, sample_envs=16):
    """Oracle port of the reference decode step on the host cores: one S=1
    step of ``sample_envs`` envs whose caches hold U[64,4096] random slots,
    repeated for about ``seconds``."""
    from oracle import decoder as odec

    threads = _host_threads()
    dec = _oracle_decoder(0)
    rng = np.random.default_rng(7)
    lens = rng.integers(LEN_LO, LEN_HI + 1, size=sample_envs)
    sess = odec.DecodeSessionOracle(dec, sample_envs)
    for li in range(LAYERS):
        sess.k[li] = [rng.standard_normal((L, KV_HEADS, HEAD_DIM)) for L in lens]
        sess.v[li] = [rng.standard_normal((L, KV_HEADS, HEAD_DIM)) for L in lens]
    sess.lengths = lens.astype(np.int64)
    emb = rng.standard_normal((sample_envs, 1, HIDDEN))
    steps, t0 = 0, time.perf_counter()
    while True:
        sess.forward(emb, [1] * sample_envs)
        steps += 1
        el = time.perf_counter() - t0
        if el >= seconds:
            break
    return {"value": round(sample_envs * steps / el, 3), "unit": "env-steps/s", "cores": threads,
            "kind": "port",
            "sample": f"{steps} decode steps of {sample_envs} envs (2 layers, float64 numpy oracle restating "
                      f"FlexDecodeSession.forward), cache lengths U[64,4096], {el:.1f} s"}


def train_cpu_baseline(seconds=15.0, row_len=2048, layers=1):
    """The reference's CPU training path (dense additive segment-causal mask +
    restarting position ids through the transformers stack, models/base.py:
    962-969, 1204-1236), fp32, forward + backward of the TD loss, on a reduced
    instance: ``layers`` of the 28-layer Qwen3-0.6B stack and one row of
    ``row_len`` tokens. tokens/s is scaled by layers/28 to a full-depth
    figure (marked as extrapolated)."""
    import torch

    from mouse_core_b200.backbone import Qwen3Backbone
    from mouse_core_b200.packing import flat_sequence_causal_mask, flat_sequence_position_ids
    from mouse_core_b200.train import ActionValueHead, td_loss

    threads = _host_threads()
    torch.manual_seed(0)
    bb = Qwen3Backbone(hidden_dim=HIDDEN, num_layers=layers, num_heads=HEADS, num_key_value_heads=KV_HEADS,
                       head_dim=HEAD_DIM, intermediate_size=INTER,
                       rope_parameters={"rope_type": "default", "rope_theta": ROPE_THETA}).float()
    emb = torch.nn.Embedding(VOCAB, HIDDEN)
    head = ActionValueHead(HIDDEN, 4)
    segs = train_row_segments(0, rows=1, row_len=row_len)[0]
    r = {k: torch.from_numpy(v) for k, v in train_row_host(100, segs).items()}
    steps, t0 = 0, time.perf_counter()
    while True:
        mask = flat_sequence_causal_mask(sequence_ids=r["sequence_ids"], dtype=torch.float32)
        pos = flat_sequence_position_ids(r["sequence_ids"])
        h = bb(emb(r["token_ids"])[None], attention_mask=mask, position_ids=pos)[0]
        loss = td_loss(head(h), r["q_target"], r["action"], r["reward"], r["done"], r["sequence_ids"])
        loss.backward()
        steps += 1
        el = time.perf_counter() - t0
        if el >= seconds:
            break
    per_layer = row_len * steps / el * layers
    return {"value": round(per_layer / TRAIN_LAYERS, 3), "unit": "tokens/s", "cores": threads,
            "kind": "port", "per_layer_tokens_per_s": round(per_layer, 1),
            "sample": f"{steps} fwd+bwd passes of one {row_len}-token row (segments {segs}) through {layers} "
                      f"layer(s), fp32 dense-mask SDPA path, {el:.1f} s; value extrapolated to 28 layers"}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return None
    if args.train:
        base = train_cpu_baseline(seconds=max(args.cpu_seconds, 5.0))
        return {"impl": "reference", "metric": "tokens/s in packed DQN training (fwd+bwd+AdamW)",
                "value": base["value"], "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
                "dtype": "f32", "data": "synthetic", "config": train_config(world, args.train_rows),
                "cpu_baseline": base, "e2e": {"value": base["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0,
                                              "d2h_bytes_per_step": 0}}
    per_step = max(args.cpu_seconds / max(args.steps + args.warmup, 1), 1.0)
    base = cpu_baseline(seconds=per_step * args.steps)
    return {"impl": "reference", "metric": "env-steps/s in cached batched decode", "value": base["value"],
            "unit": "env-steps/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f64",
            "data": "synthetic", "config": workload_config(world), "cpu_baseline": base,
            "e2e": {"value": base["value"], "unit": "env-steps/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-packed", action="store_true", help="skip the packed-attention secondary metric")
    ap.add_argument("--packed-only", action="store_true", help="only time the packed-attention kernels")
    ap.add_argument("--packed-rows", type=int, default=8, help="16384-token rows in the packed stream")
    ap.add_argument("--prefill-only", action="store_true", help="only time the paged prefill attention")
    ap.add_argument("--envs", type=int, default=ENVS, help="envs per GPU (256 is the benchmark workload; "
                    "smaller values only for profiling captures)")
    ap.add_argument("--train", action="store_true", help="time the packed DQN training step instead of decode")
    ap.add_argument("--train-rows", type=int, default=TRAIN_ROWS, help="16384-token rows per training step")
    ap.add_argument("--no-train", action="store_true", help="leave the training object out of the decode line")
    ap.add_argument("--no-extra", action="store_true",
                    help="leave the large-batch and GRPO objects out of the decode line")
    ap.add_argument("--extra-steps", type=int, default=5,
                    help="timed steps of the large-batch and GRPO objects in the decode line")
    ap.add_argument("--train-steps", type=int, default=5,
                    help="timed steps of the training object in the decode line (its warm-up is --warmup)")
    ap.add_argument("--large-batch", action="store_true",
                    help="time large-batch decode (Llama-3.2-1B arch, 512 envs/GPU, hd 64) instead")
    ap.add_argument("--lb-envs", type=int, default=LB["envs"], help="envs per GPU for --large-batch")
    ap.add_argument("--grpo", action="store_true",
                    help="time GRPO branch decode (8-layer Qwen3-0.6B arch, 64 roots x 16 forked branches)")
    ap.add_argument("--grpo-roots", type=int, default=GR["roots"], help="roots per GPU for --grpo")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    globals()["ENVS"] = args.envs
    if args.large_batch and args.impl == "ours":
        out = run_large_batch(args)
    elif args.grpo and args.impl == "ours":
        out = run_grpo(args)
    elif args.train and args.impl == "ours":
        out = run_train(args)
    elif args.prefill_only:
        import torch

        out = prefill_attention_metric(torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0"))),
                                       reps=args.steps)
    elif args.packed_only:
        import torch

        out = packed_attention_metric(torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0"))),
                                      reps=args.steps, rows=args.packed_rows)
    else:
        out = run_reference(args) if args.impl == "reference" else run_ours(args)
    if out is not None:
        print(json.dumps(out), flush=True)


if __name__ == "__main__":
    main()
