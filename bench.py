"""Batch-32 decode benchmark of the BitNet-2B-shaped model on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

One process per GPU (torchrun for N > 1, NCCL only for the barrier and the
max-over-ranks of the timings; the decode step itself has no collective).
Each rank decodes its own 32 sequences with replicated weights (weak scaling).

Workload (per rank): seeded random-init 2B-4T-shaped model (30 layers, hidden
2560, FFN 6912, 20/5 heads, vocab 128256), 32 prompts of 64 uniform random
token ids, greedy decode of 128 new tokens into a bf16 KV cache of 2048 rows,
the whole decode step captured in one CUDA graph.  The timed region replays
the step K times; after every 128 generated tokens the positions return to 64
(the prompt's KV rows stay valid), so every timed step decodes at a context of
64..192 tokens exactly as the 128-token generation does.  The step streams
~1.26 GB of weights (> 126 MB L2), so no L2 flush is needed between steps.

Line keys: value = generated tokens/s over all ranks (device-timed, inputs
resident); e2e = the same through Batch32Generator.generate_streaming-style
host I/O (ids H2D from pinned memory and new ids D2H every step); roofline =
the dominant kernel against the measured HBM peak; cpu_baseline = the CPU
oracle (a restatement of the reference's CPU path) on this host's cores.
"""

from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "bitnet-tt_b200"))

import numpy as np  # noqa: E402
import torch  # noqa: E402

METRIC = "batch-32 decode tok/s (BitNet-2B shape)"
METRIC_C1 = "batch-1 decode tok/s (BitNet-2B shape)"
REF_SINGLE_USER_TOK_S = 74.04  # reference README: packed_ternary decode, 1 user, 128 tokens, p150a
FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1590.0

# DRAM bytes per launch (dram__bytes_read.sum + dram__bytes_write.sum) from one ncu
# capture of each kernel class inside the batch-32 decode step (caches flushed before
# the captured launch); profiles/decode_step_dram_bytes_b32.md has the capture.  Used
# only at that batch; None where no capture of the current kernel exists.
NCU_TRAFFIC_BATCH = 32
# Decode attention: DRAM bytes / algorithmic bytes of one launch at config-4 contexts
# (359,606,784 / 353,400,320; profiles/gqa_decode_attention_config4_64seq.md).  Every
# K/V row is read once, so the traffic of a launch scales with the keys it reads.
NCU_TRAFFIC_RATIO: dict[str, float] = {"attention": 359606784.0 / 353400320.0}
NCU_TRAFFIC_BYTES: dict[str, float | None] = {
    "bitlinear_qkv": 2611168.0,
    "bitlinear_o": 1955136.0,
    "bitlinear_gate_up": 8998432.0,
    "bitlinear_down": 4879616.0,
    "act_quant": 186432.0,
    "lm_head": 657273280.0,
}

# Kernel classes timed by kernel_rooflines, grouped by the kernel (template
# instance) that runs them; the roofline line reports the group with the most
# time per decode step.
KERNEL_GROUPS = {
    "bitlinear_tc_kernel<residual> (o_proj, down)": ("bitlinear_o", "bitlinear_down"),
    "bitlinear_tc_kernel<relu2> (gate_up)": ("bitlinear_gate_up",),
    "bitlinear_tc_kernel<none> (qkv)": ("bitlinear_qkv",),
    "act_quant_row_kernel": ("act_quant",),
    "gqa_decode_kernel": ("attention",),
    "lm_head (tile_hidden + lm_head_tc + argmax_reduce)": ("lm_head",),
    "decode_layers_kernel": ("decode_layers",),
}


def roofline_groups(rl: dict, hbm_peak: float) -> dict:
    out = {}
    for name, members in KERNEL_GROUPS.items():
        m = [rl[k] for k in members if k in rl]
        if not m:
            continue
        ms = sum(x["ms_per_step"] for x in m)
        counts = [x["ms_per_step"] * 1e3 / x["us_per_launch"] for x in m]
        byts = sum(x["bytes_per_launch"] * c for x, c in zip(m, counts))
        n = sum(counts)
        gbs = byts / (ms * 1e-3) / 1e9
        traffic = None
        if all(x["traffic"] is not None for x in m):
            traffic = sum(x["traffic"] * c for x, c in zip(m, counts)) / n
        out[name] = {"ms_per_step": ms, "launches_per_step": n, "bytes_per_launch": byts / n,
                     "us_per_launch": ms * 1e3 / n, "achieved_gbs": gbs, "frac": gbs / hbm_peak, "traffic": traffic}
    return out


def parse() -> argparse.Namespace:
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--workload", choices=["config0", "config1", "config2", "config4"], default="config2",
                   help="config2: 32 sequences per GPU, 64-token prompts (weak scaling, the headline); config0: one "
                        "fused BitLinear [32,2560]->[32,6912]; config1: batch-1 decode, 16-token prompt; config4: "
                        "--sequences split over the GPUs, ragged contexts U[128, 4096], 256 new tokens (strong scaling)")
    p.add_argument("--sequences", type=int, default=256, help="config4: sequences over all GPUs")
    p.add_argument("--steps", type=int, default=1024)
    p.add_argument("--warmup", type=int, default=8)
    p.add_argument("--impl", choices=["b200", "reference"], default="b200")
    p.add_argument("--batch", type=int, default=32)
    p.add_argument("--prompt-len", type=int, default=None, help="default 64 (config2) / 16 (config1)")
    p.add_argument("--new-tokens", type=int, default=None, help="default 128 (config2) / 256 (config4)")
    p.add_argument("--max-seq-len", type=int, default=None, help="default 2048 (config2) / 4352 (config4)")
    p.add_argument("--layers", type=int, default=30)
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--e2e-steps", type=int, default=256)
    p.add_argument("--cpu-baseline-steps", type=int, default=2, help="0 disables the CPU baseline")
    p.add_argument("--ref-budget-s", type=float, default=60.0, help="timed CPU work of --impl reference")
    p.add_argument("--prefill-len", type=int, default=512,
                   help="config 3: time a batched prefill of --batch prompts of this length (0: skip)")
    p.add_argument("--prefill-only", action="store_true",
                   help="print only the config-3 prefill measurement (one GPU; for launch lists and captures)")
    p.add_argument("--prefill-reps", type=int, default=3)
    p.add_argument("--decode-path", choices=["per-op", "persistent"], default="per-op",
                   help="per-op: 9 launches per layer; persistent: every layer in one launch")
    p.add_argument("--clock-log", default=None,
                   help="directory for the nvidia-smi clock samples (default: a temporary directory)")
    p.add_argument("--vocab-shard", action="store_true",
                   help="with N > 1: split the lm_head by vocabulary rows over the ranks (two NCCL gathers per step)")
    return p.parse_args()


def peaks() -> tuple[float, float, str]:
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, FALLBACK_BF16_TFLOPS, "fallback"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 100 ms while running."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int, log_dir: str | None = None):
        self.gpu = gpu_index
        self.proc = None
        d = log_dir or os.path.join(tempfile.gettempdir(), f"bitnet_bench_{os.getpid()}")
        self.path = os.path.join(d, f"clocks_rank{gpu_index}.csv")

    def __enter__(self):
        os.makedirs(os.path.dirname(self.path), exist_ok=True)
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=self.f, stderr=subprocess.DEVNULL)
            time.sleep(0.3)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.15)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            self.f.close()

    def summary(self) -> dict:
        out = {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        try:
            rows = [r.split(",") for r in open(self.path).read().strip().splitlines() if r.strip()]
        except Exception:
            return out
        rows = [[c.strip() for c in r] for r in rows if len(r) >= 9]
        if not rows:
            return out
        power = [float(r[3]) for r in rows if r[3].replace(".", "", 1).isdigit()]
        thr = (max(power) * 0.5) if power else 0.0
        loaded = [r for r in rows if r[3].replace(".", "", 1).isdigit() and float(r[3]) >= thr] or rows
        out["sm_mhz"] = statistics.median(float(r[1]) for r in loaded)
        out["sm_max_mhz"] = max(float(r[2]) for r in rows)
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = set()
        for r in loaded:
            for name, v in zip(names, r[5:9]):
                if v.lower() == "active":
                    reasons.add(name)
        out["reasons"] = sorted(reasons)
        out["samples"] = len(loaded)
        return out


def dist_setup(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180),
                                device_id=torch.device("cuda", local))
    return world, rank, local


def allreduce_max(x: float, world: int, device) -> float:
    if world == 1:
        return x
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world: int) -> None:
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def model_config(args):
    from bitnet_tt.config import BitNet2B4TConfig

    return BitNet2B4TConfig(num_layers=args.layers)


# ---------------------------------------------------------------------------
# CPU side: the oracle (restatement of the reference's CPU path)
# ---------------------------------------------------------------------------
def workload_prompts(args, cfg, rank: int = 0) -> np.ndarray:
    """The prompt ids rank `rank` decodes in configs 1 and 2 (both arms use them)."""
    rng = np.random.default_rng(args.seed * 1000 + rank)
    return rng.integers(0, cfg.vocab_size, size=(args.batch, args.prompt_len))


def workload_config(args, world: int, b: int, lens, c4: bool, parallelism: str) -> dict:
    """The `config` object of the JSON line; identical in both arms apart from
    `parallelism`."""
    return {
        "workload": (f"config4: {args.sequences} sequences split over {world} GPU(s), ragged contexts "
                     f"U[128, 4096], {args.new_tokens} new tokens, bf16 KV cache {args.max_seq_len}, "
                     "CUDA graph") if c4 else
                    ("config1: batch-1 greedy decode, BitNet-2B-4T shape, 16-token prompt, 128 new "
                     "tokens, CUDA graph") if args.workload == "config1" else
                    ("config2: batch-32 greedy decode, BitNet-2B-4T shape, 64-token prompts, "
                     "128 new tokens, bf16 KV cache 2048, CUDA graph"),
        "batch_per_gpu": b, "global_batch": b * world,
        "prompt_len": (f"ragged, rank 0 mean {float(np.mean(lens)):.0f}, max {int(np.max(lens))}" if c4
                       else args.prompt_len),
        "new_tokens": args.new_tokens, "layers": args.layers, "parallelism": parallelism,
        "decode_path": args.decode_path,
        "lm_head": f"vocab-sharded over {world} ranks (NCCL gathers)" if args.vocab_shard and world > 1
        else "replicated",
        "l2": "inputs larger than L2 (1.26 GB weights streamed per step)",
    }


def cpu_decode_sample(args, steps: int, budget_s: float | None = None, warm: int = 1) -> dict:
    """Build the CPU oracle of the same model, prefill the same prompts as the
    GPU arm (rank 0's), then time `steps` batch decode steps (`warm` untimed
    steps first) from the end of the prompts."""
    from bitnet_tt.utils.weights import synthetic_state_dict
    from oracle.model import OracleBitNet

    torch.set_num_threads(os.cpu_count() or 1)
    cfg = model_config(args)
    sd = synthetic_state_dict(cfg, args.seed, device="cpu")
    steps = min(steps, args.new_tokens)  # positions stay within the workload's generation length
    ctx = args.prompt_len + max(1, warm) + steps + 1
    o = OracleBitNet(cfg, sd, max_len=ctx, quant="torch")
    b = args.batch
    caches = o.new_cache(b)
    t0 = time.perf_counter()
    ids, _ = o.prefill(workload_prompts(args, cfg), caches)  # untimed: fills KV rows 0 .. prompt_len-1
    prefill_s = time.perf_counter() - t0
    pos = torch.full((b,), args.prompt_len, dtype=torch.int32)
    for _ in range(max(1, warm)):  # untimed
        ids, _ = o.step(ids, pos, caches)
        pos = pos + 1
    done, t0 = 0, time.perf_counter()
    while done < steps:
        ids, _ = o.step(ids, pos, caches)
        pos = pos + 1
        done += 1
        if budget_s is not None and time.perf_counter() - t0 > budget_s:
            break
    dt = time.perf_counter() - t0
    return {"tok_s": b * done / dt, "steps": done, "seconds": dt, "threads": torch.get_num_threads(),
            "prefill_s": prefill_s}


def run_reference(args) -> None:
    world, rank = int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    want = max(1, args.steps)
    # the timed steps stop after --ref-budget-s seconds of CPU work (each step is ~1 s on 16 threads)
    r = cpu_decode_sample(args, want, budget_s=args.ref_budget_s, warm=args.warmup)
    sample = (f"{r['steps']} of {want} requested batch-{args.batch} decode steps of the full "
              f"{args.layers}-layer model on the CPU oracle ({r['threads']} threads), after a prefill of the "
              f"same {args.batch} x {args.prompt_len} prompt ids as the B200 arm ({r['prefill_s']:.1f} s, untimed) "
              f"and {args.warmup} untimed steps")
    c1 = args.workload == "config1"
    line = {
        "impl": "reference", "metric": METRIC_C1 if c1 else METRIC, "value": r["tok_s"], "unit": "tok/s",
        "n_gpus": world, "steps": r["steps"], "warmup": args.warmup, "ms_per_step": 1000.0 * r["seconds"] / r["steps"],
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "int8xternary->int32 (bf16 act/KV, bf16 lm_head)",
        "data": "synthetic (seeded random-init weights, uniform random prompt ids)",
        "config": workload_config(args, world, args.batch, [args.prompt_len], False, "CPU oracle, rank 0"),
        "cpu_baseline": {"value": r["tok_s"], "unit": "tok/s", "cores": r["threads"], "kind": "port",
                         "sample": sample},
        "e2e": {"value": r["tok_s"], "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# GPU side
# ---------------------------------------------------------------------------
def graph_of(fn, device):
    side = torch.cuda.Stream(device=device)
    side.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(side):
        fn()
    torch.cuda.current_stream(device).wait_stream(side)
    torch.cuda.synchronize(device)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        fn()
    torch.cuda.synchronize(device)
    return g


def time_graph(g, reps: int) -> float:
    """Average ms per replay (events on the replay stream, synchronize on both sides)."""
    torch.cuda.synchronize()
    g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        g.replay()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / reps


def kernel_rooflines(gen, args, hbm_peak: float) -> dict:
    """Time each kernel class in isolation (a graph of one launch per layer, so the
    weights streamed exceed L2) and relate algorithmic bytes to the HBM peak."""
    from bitnet_tt import _lib

    st, m, cfg = gen.state, gen.model, gen.config
    b = st.batch
    h, f, v = cfg.hidden_size, cfg.intermediate_size, cfg.vocab_size
    qkv_n = st.qkv.shape[1]
    res: dict[str, dict] = {}

    def entry(name, fn, launches_per_replay, bytes_per_launch, count_per_step):
        g = graph_of(fn, m.device)
        ms = time_graph(g, 20)
        per = ms / launches_per_replay
        gbs = bytes_per_launch / (per * 1e-3) / 1e9
        traffic = NCU_TRAFFIC_BYTES.get(name) if b == NCU_TRAFFIC_BATCH else None
        if name in NCU_TRAFFIC_RATIO:
            traffic = bytes_per_launch * NCU_TRAFFIC_RATIO[name]
        res[name] = {"us_per_launch": per * 1e3, "bytes_per_launch": bytes_per_launch, "achieved_gbs": gbs,
                     "frac": gbs / hbm_peak, "ms_per_step": per * count_per_step, "traffic": traffic}
        del g

    nl = len(m.layers)
    eps = cfg.rms_norm_eps
    _lib.act_quant(st.hidden, m.layers[0].input_layernorm.weight, eps, st.act_h)
    _lib.act_quant(st.mid, m.layers[0].mlp.ffn_sub_norm.weight, eps, st.act_f)
    torch.cuda.synchronize()
    out_h = torch.empty_like(st.hidden)
    out_f = torch.empty_like(st.mid)
    out_qkv = torch.empty_like(st.qkv)
    # algorithmic bytes of one bitlinear_q launch: packed W + int8 q + bf16 y (+ bf16 residual read)
    wbytes = lambda n, k: n * k // 4  # noqa: E731
    entry("bitlinear_qkv", lambda: [L.self_attn.qkv_proj.forward_into(st.act_h, b, out_qkv) for L in m.layers], nl,
          wbytes(qkv_n, h) + b * h + 2 * b * qkv_n, nl)
    entry("bitlinear_o", lambda: [L.self_attn.o_proj.forward_into(st.act_h, b, out_h, residual=st.hidden)
                                  for L in m.layers], nl, wbytes(h, h) + b * h + 4 * b * h, nl)
    entry("bitlinear_gate_up", lambda: [L.mlp.gate_up_proj.forward_into(st.act_h, b, out_f) for L in m.layers], nl,
          wbytes(2 * f, h) + b * h + 2 * b * f, nl)
    entry("bitlinear_down", lambda: [L.mlp.down_proj.forward_into(st.act_f, b, out_h, residual=st.hidden)
                                     for L in m.layers], nl, wbytes(h, f) + b * f + 4 * b * h, nl)
    entry("act_quant", lambda: [_lib.act_quant(st.hidden, L.input_layernorm.weight, eps, st.act_h)
                                for L in m.layers], nl, 2 * b * h + b * h + 2 * h, 4 * nl)
    ctx = st.positions.float().mean().item() + 1
    kv_bytes = int(b * ctx * cfg.num_key_value_heads * cfg.head_dim * 2 * 2)
    pos_save = st.positions.clone()
    entry("attention", lambda: [L.self_attn.decode_attention(st.qkv, st.positions, st.rope_cos, st.rope_sin, c,
                                                              st.attn, st.max_ctx, st.attn_ws)
                                for L, c in zip(m.layers, st.caches)], nl,
          kv_bytes + 2 * b * qkv_n + 2 * b * h, nl)
    if gen.persistent:
        # every layer in one persistent launch: all packed weights + the KV rows read + activations
        layer_w = wbytes(qkv_n, h) + wbytes(h, h) + wbytes(2 * f, h) + wbytes(h, f)
        entry("decode_layers", lambda: st.plan.run(), 1, nl * (layer_w + kv_bytes + 2 * b * (qkv_n + 3 * h + 2 * f)), 1)
    ws = st.argmax_ws
    ids = torch.empty_like(st.ids)
    entry("lm_head", lambda: m.lm_head_argmax(st.normed, ws, ids), 1, 2 * v * h + 2 * b * h, 1)  # 3 launches
    st.positions.copy_(pos_save)
    torch.cuda.synchronize()
    return res


def prefill_measure(model, args, device, reps: int = 3) -> dict:
    """one batched prefill of --batch prompts of --prefill-len
    uniform random ids through the full model (TTFT).  device_ms: CUDA events
    around the prefill enqueue (prompt ids uploaded inside); ttft_ms: host wall
    clock from the prompt table on the host to the first generated ids on the
    host.  The BitLinear and attention classes are then timed alone (graphs of
    the prefill's own launches over all layers) for their tensor-pipe rates."""
    from bitnet_tt import _lib
    from bitnet_tt.inference import Batch32Generator

    cfg = model.config
    b, plen = args.batch, args.prefill_len
    n = b * plen
    gen = Batch32Generator(model, batch_size=b, max_seq_len=plen + 64)
    gen.set_context_limit(plen + 1)
    prompts = np.random.default_rng(args.seed + 17).integers(0, cfg.vocab_size, size=(b, plen))
    gen.prefill(prompts)  # allocations, decode-graph capture, first launches
    torch.cuda.synchronize(device)
    if _lib.last_device_status()[0] != 0:
        raise RuntimeError(f"device status {_lib.last_device_status()} after prefill warm-up")
    dev_ms, wall_ms = [], []
    for _ in range(reps):
        gen.reset()
        torch.cuda.synchronize(device)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        gen._prefill_batched(prompts)
        e1.record()
        torch.cuda.synchronize(device)
        dev_ms.append(e0.elapsed_time(e1))
    for _ in range(reps):
        gen.reset()
        torch.cuda.synchronize(device)
        t0 = time.perf_counter()
        gen._prefill_batched(prompts)
        first = gen.state.ids.cpu()
        wall_ms.append((time.perf_counter() - t0) * 1e3)
    assert first.numel() == b

    pb, st, m = gen.prefill_buffers, gen.state, gen.model
    h, f = cfg.hidden_size, cfg.intermediate_size
    nq, nkv, d = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim
    qkv_n = (nq + 2 * nkv) * d
    nl = len(m.layers)
    lin_ops = 2 * n * nl * (qkv_n * h + h * nq * d + 2 * f * h + h * f)
    g = graph_of(lambda: [(L.self_attn.qkv_proj.forward_into(pb.act_h, n, pb.qkv),
                           L.self_attn.o_proj.forward_into(pb.act_h, n, pb.attn),
                           L.mlp.gate_up_proj.forward_into(pb.act_h, n, pb.mid),
                           L.mlp.down_proj.forward_into(pb.act_f, n, pb.hidden)) for L in m.layers], device)
    lin_ms = time_graph(g, 3)
    del g
    att_flops = 4 * d * b * nq * nl * plen * (plen + 1) // 2  # QK^T and PV over the causal triangle
    g = graph_of(lambda: [_lib.attention_prefill(pb.q, c.key_cache, c.value_cache, b, plen, nq, nkv,
                                                 d ** -0.5, pb.attn) for c in st.caches], device)
    att_ms = time_graph(g, 3)
    del g
    gen.release_trace()
    gen.release_prefill_buffers()
    int8_peak = 2 * FALLBACK_BF16_TFLOPS
    bf16_peak = FALLBACK_BF16_TFLOPS
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as fh:
            bf16_peak = float(json.load(fh)["bf16_tflops"])
            int8_peak = 2 * bf16_peak
    except (OSError, KeyError, ValueError):
        pass
    dev = statistics.median(dev_ms)
    return {
        "workload": f"config3: batched prefill of {b} prompts x {plen} uniform random ids, {nl} layers",
        "tokens": n, "ttft_ms": round(statistics.median(wall_ms), 3), "device_ms": round(dev, 3),
        "prompt_tok_s": round(n / (dev / 1e3), 1),
        "bitlinear": {"ms": round(lin_ms, 3), "int_ops": lin_ops, "achieved_tops": round(lin_ops / lin_ms / 1e9, 1),
                      "peak_tops": int8_peak, "frac": round(lin_ops / lin_ms / 1e9 / int8_peak, 4),
                      "peak_kind": "int8 dense = 2 x measured bf16 GEMM burst"},
        "attention": {"ms": round(att_ms, 3), "flops": att_flops, "achieved_tflops": round(att_flops / att_ms / 1e9, 1),
                      "peak_tflops": bf16_peak, "frac": round(att_flops / att_ms / 1e9 / bf16_peak, 4),
                      "peak_kind": "measured bf16 GEMM burst"},
    }


def run_config0(args) -> None:
    """one fused BitLinear (RMSNorm + int8 act-quant + ternary
    contraction + scale) x [32, 2560] bf16 -> y [32, 6912] bf16, W ternary with
    P(0) = 0.4, scale 0.02.  The timed unit is one call (act-quant launch + BitLinear
    launch) replayed from a CUDA graph over 40 weight copies (177 MB > L2, so every
    call streams its 4.4 MB of weights from HBM).  e2e: the public Linear call with
    the input from pinned host memory and the output read back every call.  CPU
    baseline: the oracle's fused BitLinear (NumPy) on the host cores."""
    from bitnet_tt import _lib
    from bitnet_tt.layers.bitlinear import Linear
    from oracle import bitlinear as ob

    if args.gpus != 1:
        raise SystemExit("config0 runs on one GPU")
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    hbm_peak, _, peak_kind = peaks()
    m, k, n, copies = 32, 2560, 6912, 40
    g = torch.Generator().manual_seed(args.seed)
    x = torch.randn((m, k), generator=g).to(torch.bfloat16)
    gamma = (1 + 0.1 * torch.randn(k, generator=g)).to(torch.bfloat16)
    rng = np.random.default_rng(args.seed)
    wq = [rng.choice(np.array([-1, 0, 1], np.int8), size=(n, k), p=[0.3, 0.4, 0.3]) for _ in range(copies)]
    ws = [_lib.pack_ternary(torch.from_numpy(w).to(dev)) for w in wq]
    xd, gd = x.to(dev), gamma.to(dev)
    bufs = _lib.ActBuffers(m, k, dev)
    y = torch.empty((m, n), dtype=torch.bfloat16, device=dev)
    seg = _lib.Segments.make([n], [0.02])

    def calls():
        for i in range(copies):
            _lib.act_quant(xd, gd, 1e-5, bufs)
            _lib.bitlinear_q(bufs, m, k, ws[i], n, seg, _lib.EPI_NONE, None, y)

    graph = graph_of(calls, dev)
    for _ in range(args.warmup):
        graph.replay()
    reps = max(1, args.steps // copies)
    torch.cuda.synchronize(dev)
    with ClockSampler(0, args.clock_log) as clocks:
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            graph.replay()
        e1.record()
        torch.cuda.synchronize(dev)
    us = e0.elapsed_time(e1) * 1e3 / (reps * copies)
    algo = n * k // 4 + 2 * m * k + 2 * m * n  # packed W + bf16 x + bf16 y
    ops = 2 * m * n * k
    # parity of the timed call against the oracle (last weight copy)
    ref = ob.bitlinear(x.float().numpy(), gamma.float().numpy(), 1e-5, wq[-1], [n], [0.02])
    exact = bool(np.array_equal(y.float().cpu().numpy(), ref["y"]))
    # e2e through the public layer: host input in, host output back, every call
    lin = Linear(k, n, dev)
    lin.load_ternary(torch.from_numpy(wq[0]).to(dev), 0.02)
    hx = x.pin_memory()
    hy = torch.empty((m, n), dtype=torch.bfloat16).pin_memory()
    for _ in range(3):
        hy.copy_(lin(hx.to(dev, non_blocking=True), norm_weight=gd, norm_epsilon=1e-5), non_blocking=True)
    torch.cuda.synchronize(dev)
    ne = 200
    t0 = time.perf_counter()
    for _ in range(ne):
        hy.copy_(lin(hx.to(dev, non_blocking=True), norm_weight=gd, norm_epsilon=1e-5), non_blocking=True)
        torch.cuda.current_stream(dev).synchronize()
    e2e_us = (time.perf_counter() - t0) * 1e6 / ne
    # CPU baseline: the oracle on this host's cores
    cpu_t = []
    xf, gf = x.float().numpy(), gamma.float().numpy()
    ob.bitlinear(xf, gf, 1e-5, wq[0], [n], [0.02])
    for _ in range(5):
        t0 = time.perf_counter()
        ob.bitlinear(xf, gf, 1e-5, wq[0], [n], [0.02])
        cpu_t.append(time.perf_counter() - t0)
    cpu_s = statistics.median(cpu_t)
    gbs = algo / (us * 1e-6) / 1e9
    line = {
        "metric": "fused BitLinear x[32,2560] -> y[32,6912] GB/s (BASELINE config 0)", "value": round(gbs, 1),
        "unit": "GB/s", "n_gpus": 1, "steps": reps * copies, "warmup": args.warmup, "us_per_call": round(us, 3),
        "ms_per_step": round(us / 1e3, 5), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "int8xternary->int32 (bf16 in/out)", "data": "synthetic (seeded x, gamma, ternary W with P(0)=0.4)",
        "config": {"workload": "config0: act-quant + tcgen05 BitLinear per call, 40 weight copies rotated (177 MB > "
                               "L2)", "algorithmic_bytes": algo, "int8_ops": ops,
                   "gops": round(ops / (us * 1e-6) / 1e9, 1), "bit_exact_vs_oracle": exact},
        "e2e": {"value": round(algo / (e2e_us * 1e-6) / 1e9, 2), "unit": "GB/s", "us_per_call": round(e2e_us, 2),
                "h2d_bytes_per_step": 2 * m * k, "d2h_bytes_per_step": 2 * m * n},
        "gpu_launches": 2 * reps * copies,
        "roofline": {"kernel": "act_quant_row_kernel + bitlinear_tc_kernel<none>", "bound": "hbm",
                     "achieved": round(gbs, 1), "peak": hbm_peak, "unit": "GB/s", "frac": round(gbs / hbm_peak, 4),
                     "traffic": None, "peak_kind": peak_kind},
        "cpu_baseline": {"value": round(algo / cpu_s / 1e9, 3), "unit": "GB/s", "cores": os.cpu_count(),
                         "kind": "port", "sample": f"median of 5 oracle calls, {cpu_s * 1e3:.1f} ms each"},
        "clocks": clocks.summary(), "device_status": _lib.last_device_status()[0],
    }
    print(json.dumps(line), flush=True)


def run_prefill_only(args) -> None:
    from bitnet_tt.model import create_model
    from bitnet_tt.utils.weights import load_weights_to_model, synthetic_state_dict

    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    cfg = model_config(args)
    model = create_model(cfg, device)
    load_weights_to_model(model, synthetic_state_dict(cfg, args.seed, device=device))
    torch.cuda.synchronize(device)
    print(json.dumps({"prefill": prefill_measure(model, args, device, reps=args.prefill_reps)}), flush=True)


def run_b200(args) -> None:
    world, rank, local = dist_setup(args)
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    from bitnet_tt import _lib
    from bitnet_tt.inference import Batch32Generator
    from bitnet_tt.model import create_model
    from bitnet_tt.utils.weights import load_weights_to_model, synthetic_state_dict

    hbm_peak, _, peak_kind = peaks()
    cfg = model_config(args)
    t_build = time.perf_counter()
    model = create_model(cfg, device)
    load_weights_to_model(model, synthetic_state_dict(cfg, args.seed, device=device))
    torch.cuda.synchronize(device)
    t_build = time.perf_counter() - t_build

    c4 = args.workload == "config4"
    if c4 and args.sequences % world != 0:
        raise SystemExit("--sequences must be a multiple of the GPU count")
    b = args.sequences // world if c4 else args.batch
    shard = args.vocab_shard and world > 1
    import torch.distributed as dist  # noqa: F811 - only used when world > 1

    gen = Batch32Generator(model, batch_size=b, max_seq_len=args.max_seq_len,
                           persistent=args.decode_path == "persistent",
                           vocab_shard_group=dist.group.WORLD if shard else None)
    if c4:
        # ragged contexts: all --sequences lengths drawn from one seeded stream, each rank takes its slice
        lens_all = np.random.default_rng(args.seed).integers(128, 4097, size=args.sequences)
        lens = lens_all[rank * b:(rank + 1) * b]
        rng = np.random.default_rng(args.seed * 1000 + rank)
        prompts = [rng.integers(0, cfg.vocab_size, size=int(n)) for n in lens]
        gen.set_context_limit(int(lens.max()) + args.new_tokens)
    else:
        lens = np.full(b, args.prompt_len)
        gen.set_context_limit(args.prompt_len + args.new_tokens)  # positions cycle within it
        prompts = workload_prompts(args, cfg, rank)
    torch.cuda.synchronize(device)
    t_pf = time.perf_counter()
    gen.prefill(prompts)
    torch.cuda.synchronize(device)
    t_pf = time.perf_counter() - t_pf
    st = gen.state
    first_pos_d = torch.from_numpy(lens.astype(np.int32)).to(device)

    produced = 0  # tokens generated since the last position reset

    def step():
        nonlocal produced
        if produced == args.new_tokens:
            st.positions.copy_(first_pos_d)  # back to the end of each prompt: contexts stay within the cache
            produced = 0
        gen.step()
        produced += 1

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(device)
    st_status = _lib.last_device_status()
    if st_status[0] != 0:
        raise RuntimeError(f"device status {st_status} after warm-up")

    # ---- device-timed decode ------------------------------------------------
    barrier(world)
    torch.cuda.synchronize(device)
    with ClockSampler(local, args.clock_log) as clocks:
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            step()
        e1.record()
        torch.cuda.synchronize(device)
    barrier(world)
    ms = e0.elapsed_time(e1)
    ms_max = allreduce_max(ms, world, device)
    value = world * b * args.steps / (ms_max / 1000.0)

    # ---- end to end through the streaming API pattern (host ids in / out) ----
    host_in = torch.empty(b, dtype=torch.int32, pin_memory=True)
    host_out = torch.empty(b, dtype=torch.int32, pin_memory=True)
    host_out.copy_(st.ids)
    barrier(world)
    torch.cuda.synchronize(device)
    t0 = time.perf_counter()
    for _ in range(args.e2e_steps):
        host_in.copy_(host_out)
        st.ids.copy_(host_in, non_blocking=True)
        step()
        host_out.copy_(st.ids, non_blocking=True)
        torch.cuda.current_stream(device).synchronize()
    e2e_s = allreduce_max(time.perf_counter() - t0, world, device)
    e2e_value = world * b * args.e2e_steps / e2e_s

    # ---- per-kernel rooflines (rank 0) ----------------------------------------
    rl = kernel_rooflines(gen, args, hbm_peak) if rank == 0 else {}
    launches_per_step = gen.launches_per_step
    gen.release_trace()
    prefill = None
    if rank == 0 and args.prefill_len > 0 and not shard:
        del gen
        torch.cuda.empty_cache()
        prefill = prefill_measure(model, args, device)
    status = _lib.last_device_status()

    cpu = None
    if rank == 0 and world == 1 and args.cpu_baseline_steps > 0:
        gen = None
        del gen, model
        torch.cuda.empty_cache()
        r = cpu_decode_sample(args, args.cpu_baseline_steps)
        cpu = {"value": r["tok_s"], "unit": "tok/s", "cores": r["threads"], "kind": "port",
               "sample": f"{r['steps']} batch-{b} decode steps of the full {args.layers}-layer model on the CPU "
                         f"oracle after a prefill of the same prompt ids ({r['prefill_s']:.1f} s, untimed) and "
                         f"1 warm step (context {args.prompt_len + 1}..)"}

    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()
    if rank != 0:
        return

    groups = roofline_groups(rl, hbm_peak) if rl else {}
    dominant = max(groups, key=lambda k: groups[k]["ms_per_step"]) if groups else None
    roof = None
    if dominant:
        d = groups[dominant]
        roof = {"kernel": dominant, "bound": "hbm", "achieved": round(d["achieved_gbs"], 1),
                "peak": hbm_peak, "unit": "GB/s", "frac": round(d["frac"], 4), "traffic": d["traffic"],
                "peak_kind": peak_kind}
    launches = args.steps * launches_per_step
    # Whole-step roofline: every byte a decode step must read once (2-bit weights,
    # bf16 lm_head, the KV rows of the contexts, ~1 MB of activations ignored).
    hcfg = model_config(args)
    h_, f_ = hcfg.hidden_size, hcfg.intermediate_size
    qkv_ = (hcfg.num_attention_heads + 2 * hcfg.num_key_value_heads) * hcfg.head_dim
    w_layer = (qkv_ * h_ + h_ * hcfg.num_attention_heads * hcfg.head_dim + 2 * f_ * h_ + h_ * f_) // 4
    ctx_mean = float(lens.mean()) + (args.new_tokens + 1) / 2.0  # positions cycle len+1 .. len+new (rank 0)
    kv_step = b * ctx_mean * 2 * hcfg.num_key_value_heads * hcfg.head_dim * 2 * hcfg.num_layers
    step_bytes = hcfg.num_layers * w_layer + 2 * hcfg.vocab_size * h_ + kv_step
    step_s = ms_max / args.steps / 1000.0
    step_roof = {"bytes_per_step": int(step_bytes), "ternary_weight_bytes": hcfg.num_layers * w_layer,
                 "lm_head_bytes": 2 * hcfg.vocab_size * h_, "kv_bytes": int(kv_step),
                 "achieved_gbs": round(step_bytes / step_s / 1e9, 1), "peak": hbm_peak, "unit": "GB/s",
                 "frac": round(step_bytes / step_s / 1e9 / hbm_peak, 4), "peak_kind": peak_kind}
    line = {
        "metric": METRIC_C1 if args.workload == "config1" else METRIC, "value": round(value, 1), "unit": "tok/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_max / args.steps, 4), "higher_is_better": True,
        "scaling": "strong" if c4 else "weak",
        # the reference publishes one decode rate: single-user, 128 tokens, on a Tenstorrent p150a
        "vs_baseline": round(value / REF_SINGLE_USER_TOK_S, 2) if args.workload == "config1" else None,
        "dtype": "int8xternary->int32 (bf16 act/KV, bf16 lm_head)",
        "data": "synthetic (seeded random-init weights, uniform random prompt ids)",
        "config": workload_config(args, world, b, lens, c4, f"dp{world} (batch split)"),
        "timings": {"prefill_s_rank0": round(t_pf, 2), "model_build_s": round(t_build, 1)},
        "e2e": {"value": round(e2e_value, 1), "unit": "tok/s", "h2d_bytes_per_step": 4 * b,
                "d2h_bytes_per_step": 4 * b},
        "gpu_launches": launches,
        "roofline": roof,
        "step_roofline": step_roof,
        "roofline_groups": {k: {kk: (round(vv, 4) if isinstance(vv, float) else vv) for kk, vv in d.items()}
                            for k, d in groups.items()},
        "roofline_kernels": {k: {kk: (round(vv, 4) if isinstance(vv, float) else vv) for kk, vv in d.items()}
                             for k, d in rl.items()},
        "prefill": prefill,
        "cpu_baseline": cpu,
        "clocks": {k: v for k, v in clocks.summary().items()},
        "device_status": status[0],
    }
    print(json.dumps(line), flush=True)


def main() -> None:
    args = parse()
    c4 = args.workload == "config4"
    if args.workload == "config1":
        args.batch = 1
    if args.prompt_len is None:
        args.prompt_len = 16 if args.workload == "config1" else 64
    if args.new_tokens is None:
        args.new_tokens = 256 if c4 else 128
    if args.max_seq_len is None:
        args.max_seq_len = 4096 + args.new_tokens if c4 else 2048
    if c4:
        args.prefill_len = 0  # the prefill fills the ragged contexts; config 3 is measured in config2 runs
        args.cpu_baseline_steps = 0
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    if args.workload == "config0":
        run_config0(args)
    elif args.impl == "reference":
        run_reference(args)
    elif args.prefill_only:
        run_prefill_only(args)
    else:
        run_b200(args)


if __name__ == "__main__":
    main()
