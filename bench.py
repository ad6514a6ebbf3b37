"""Trie-verify step benchmark.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]

Workload (config 3): random-init 28-layer Qwen3-style decoder (hidden 3584,
28 q / 4 kv heads of 128, FFN 18944, vocab 152,064, RoPE theta 1e6, weights
~ N(0, 0.02), bf16); a 3,000-token prefix of seeded random ids, prefilled by
the engine; a 128-node trie of 4 chains of 32 with seeded shared prefixes, one
of them the model's own greedy continuation, so each verify step commits 32
tokens. A step = one verify forward over the trie + greedy choice (+ in the
e2e loop: host->device trie arrays, device->host ids, the host acceptance
walk and the KV compaction). Metric: committed tokens/s (whole job); latency
in ms_per_step. Weights (14.1 GB per step) exceed L2 (126 MB), so no flush
is needed between steps.

N > 1: one process per GPU (torchrun), independent replicas (frame streams)
with no collective on the data path; the timed region is bracketed by a
barrier and the max over ranks is reported.

--impl reference: the reference's CPU path on the host cores: whole verify
steps of its eager bf16 forward at the config-3 model size (a torch restatement,
oracle/torch_model.py), at most 20 timed steps.

The default line also carries `frame_replay`: config 5 measured in the same run
(16 frame streams per GPU, one untimed and --replay-frames timed frames each;
--replay-frames 0 leaves it out), so a run at N GPUs records frames/s at N.

--workload frame_replay [--streams S]: the multi-stream frame replay (S frame
streams per GPU, 4,096-token prompts, 256-node tries, 80 committed tokens per
frame); --warmup / --steps count frames per stream (defaults 1 / 2); metric
frames/s.

--kernel-case config1 | config2: the standalone operators of configs 1 and 2
(fp32 trie attention; RMSNorm, RoPE, SiLU*mul) at their BASELINE shapes, timed per
launch after an L2 flush, next to PyTorch eager on the host cores; one JSON line
per operator.

--kernel-case gemm_gate_up | attention: only that kernel at its config-3
shape (--warmup untimed launches, then --steps timed ones), for profiling one
kernel on a small footprint; prints one JSON line with the per-launch time.
  gemm_gate_up: the fused gate|up GEMM + SiLU*mul epilogue, 128 rows,
                two layers' packed weights (0.54 GB) used alternately.
  attention:    one layer's trie attention, 28/4 heads, 3000-key prefix,
                128-node trie, bf16.
  step_small:   the verify step of a ONE-layer decoder of config-3 width (every
                kernel of a config-3 layer plus the 152,064-row lm_head at its
                config-3 shape, about 4 GB on the device): the engine prefills
                the --prefix prompt in 128-row chunks, then runs --steps graph
                replays of the --nodes-row step; for per-kernel profiles.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

import numpy as np  # noqa: E402

PROMPT = 3000
NODES = 128
CHAIN = 32
KERNELS_PER_LAYER = 9          # qkv gemm, qkv finish, attn prefix, attn nodes, o gemm, resid, gu gemm, down gemm, resid
KERNELS_FIXED = 3              # embed+norm, lm_head gemm (+ greedy keys), greedy finalize


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None)
    ap.add_argument("--warmup", type=int, default=None)
    ap.add_argument("--impl", default="native", choices=["native", "reference"])
    ap.add_argument("--e2e-steps", type=int, default=None)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--kernel-case", default=None,
                    choices=["gemm_gate_up", "attention", "config1", "config2", "step_small"])
    ap.add_argument("--workload", default="verify_step", choices=["verify_step", "frame_replay"])
    ap.add_argument("--streams", type=int, default=16)
    ap.add_argument("--one-cuda-stream", action="store_true",
                    help="frame_replay: all frame streams' work on one CUDA stream")
    ap.add_argument("--nodes", type=int, default=NODES, help="verify_step: trie nodes (config 3: 128)")
    ap.add_argument("--prefix", type=int, default=PROMPT, help="verify_step: prompt tokens (config 3: 3000)")
    ap.add_argument("--replay-frames", type=int, default=1,
                    help="verify_step: timed frames per stream of the frame replay carried in the line (0: none)")
    ap.add_argument("--replay-streams", type=int, default=16)
    args = ap.parse_args()
    replay = args.workload == "frame_replay" and not args.kernel_case
    if args.steps is None:
        args.steps = 2 if replay else 300
    if args.warmup is None:
        args.warmup = 1 if replay else 5
    return args


def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


def profiled_traffic():
    """dram__bytes_read.sum + dram__bytes_write.sum of one gate|up GEMM launch, from the
    committed ncu summary (profiles/gemm_gate_up_config3.md), or None."""
    p = ROOT / "profiles" / "gemm_gate_up_config3.md"
    if not p.exists():
        return None
    for ln in p.read_text().splitlines():
        if ln.startswith("traffic_bytes_per_launch:"):
            return float(ln.split(":", 1)[1])
    return None


def config_block(n, nodes=NODES, prompt=PROMPT):
    name = "config3: " if (nodes, prompt) == (NODES, PROMPT) else ""
    return {"workload": f"{name}trie verify step, 28-layer 7B-class decoder, prefix {prompt}, {nodes}-node trie",
            "model": "qwen3-style random-init hidden3584 L28 H28/4 D128 F18944 V152064",
            "prefix": prompt, "trie_nodes": nodes, "committed_per_step": min(CHAIN, nodes), "global_batch": n,
            "parallelism": f"replicas{n}", "l2": "inputs larger than L2 (14.1 GB weights per step)"}


# ------------------------------------------------------------------ multi-rank helpers
def reduce_max(x: float, device) -> float:
    """The maximum of x over all ranks (x itself without a process group)."""
    import torch
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(x)
    t = torch.tensor([float(x)], device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def job_value(world: int, units_per_step: float, steps: int, ms: float) -> float:
    """Whole-job throughput: every rank processed units_per_step per step; ms is the max over ranks."""
    return world * units_per_step * steps / (ms / 1e3)


# ------------------------------------------------------------------ CPU baseline (whole steps)
def cpu_steps(steps, warmup, nodes=NODES, prompt=PROMPT, chain=CHAIN, seed=0):
    """Whole verify steps of the reference's eager path on the host cores: the full
    28-layer config-3 model (hidden 3584, 28 / 4 heads of 128, FFN 18944, vocab
    152,064) in bf16 through torch's CPU ops (oracle/torch_model.py, mode "eager":
    HF's RMSNorm, linears, RoPE, SDPA with the additive trie mask and SiLU*mul, as
    respect/decoding/verify.py:12-46 runs without the dedicated kernels), `nodes`
    trie rows over a `prompt`-token prefix. Each timed step is one complete
    forward; the metric counts the `chain` tokens the GPU step commits."""
    import torch

    from oracle import torch_model as tm
    from oracle.inputs import chain_seqs, top_up
    from respect_b200.candidates.trie import build_trie
    h, L, H, HK, D, F, V = 3584, 28, 28, 4, 128, 18944, 152064
    # all host threads (torchrun sets OMP_NUM_THREADS=1 for its workers)
    torch.set_num_threads(os.cpu_count() or 1)
    W = tm.random_weights_cpu(h, L, H, HK, D, F, V, seed=seed)
    g = torch.Generator().manual_seed(seed + 1)
    kc = [torch.randn(HK, prompt + nodes, D, generator=g).to(torch.bfloat16) for _ in range(L)]
    vc = [torch.randn(HK, prompt + nodes, D, generator=g).to(torch.bfloat16) for _ in range(L)]
    rng = np.random.default_rng(seed)
    tree = build_trie(top_up(rng, chain_seqs(rng, 4, chain, V), nodes, V))
    cfg = dict(n_heads=H, n_kv_heads=HK, head_dim=D, rms_eps=1e-6, rope_theta=1e6)
    times = []
    for i in range(warmup + steps):
        t0 = time.perf_counter()
        tm.verify_step(W, cfg, tree.tokens(), tree.parents(), tree.depths(), prompt, 0, kc, vc, mode="eager")
        if i >= warmup:
            times.append(time.perf_counter() - t0)
    t_step = sum(times) / len(times)
    threads = torch.get_num_threads()
    del W, kc, vc
    return dict(value=chain / t_step, unit="committed tokens/s", cores=threads, kind="port",
                sample=(f"{steps} whole verify steps (after {warmup} untimed) of the reference's eager path in bf16 "
                        f"on {threads} host threads (oracle/torch_model.py mode eager: the full 28-layer config-3 "
                        f"model, {nodes} trie rows vs a {prompt}-token prefix, torch CPU ops); mean step "
                        f"{t_step:.2f} s; {chain} committed tokens per step as on the GPU"),
                ms_per_step=t_step * 1e3, steps=steps, warmup=warmup)


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    # whole steps of a few seconds each: at most 20 timed and 2 untimed, so the
    # run stays within a couple of minutes on the host cores
    steps = max(1, min(args.steps, 20))
    warm = max(1, min(args.warmup, 2))
    cb = cpu_steps(steps, warm)
    line = {"metric": "committed tokens/s (trie-verify step)", "value": cb["value"], "unit": cb["unit"],
            "impl": "reference", "n_gpus": args.gpus, "steps": steps, "warmup": warm,
            "ms_per_step": cb["ms_per_step"], "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic (seeded)", "config": config_block(args.gpus),
            "cpu_baseline": {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")},
            "e2e": {"value": cb["value"], "unit": cb["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ clocks
class Clocks:
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.path = Path(tempfile.gettempdir()) / f"respect_b200_clocks_{os.getpid()}.csv"

    def __enter__(self):
        try:
            self.path.parent.mkdir(exist_ok=True)
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            self.proc.wait(timeout=10)
            self.f.close()

    def summary(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        rows = []
        for ln in self.path.read_text().splitlines():
            p = [x.strip() for x in ln.split(",")]
            if len(p) >= 9:
                rows.append(p)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


# ------------------------------------------------------------------ native arm
def run_native(args):
    import torch

    NODES, PROMPT = args.nodes, args.prefix  # noqa: N806 (config 3: 128, 3000)
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=dev)

    from oracle.inputs import top_up
    from respect_b200 import _lib
    from respect_b200.candidates.trie import build_trie
    from respect_b200.decoding.acceptance import walk
    from respect_b200.decoding.engine import DecoderConfig, DecoderWeights, VerifyEngine
    from respect_b200.kernels.gemm import linear_swiglu_packed

    cfg = DecoderConfig.baseline_7b()
    w = DecoderWeights.random(cfg, dev, seed=0)
    eng = VerifyEngine(w, max_rows=NODES, max_slots=PROMPT + 1024)
    rng = np.random.default_rng(100 + rank)
    eng.prefill(rng.integers(0, cfg.vocab, PROMPT))
    # the model's own greedy continuation (1-token steps) becomes one chain
    first = int(rng.integers(0, cfg.vocab))
    toks = [first]
    chain_n = min(CHAIN, NODES)   # the AR chain (32 tokens at config 3) fits the trie
    for t in range(chain_n):
        eng.step(np.array([toks[-1]], np.int32), np.array([-1], np.int32), np.array([0], np.int32), t, PROMPT)
        toks.append(int(eng.fetch_ids(1)[0]))
    seqs = [tuple(toks[:chain_n])]
    for _ in range(64):   # up to 3 more chains sharing a seeded prefix with it, while they fit
        if len(seqs) == 4 or chain_n < 2:
            break
        share = int(rng.integers(1, chain_n))
        cand = tuple(toks[:share]) + tuple(int(x) for x in rng.integers(0, cfg.vocab, chain_n - share))
        if len(build_trie(seqs + [cand]).nodes) <= NODES:
            seqs.append(cand)
    tree = build_trie(top_up(rng, seqs, NODES, cfg.vocab))
    assert len(tree.nodes) == NODES
    ids_d = torch.from_numpy(tree.tokens().astype(np.int32)).to(dev)
    par_d = torch.from_numpy(tree.parents()).to(dev)
    dep_d = torch.from_numpy(tree.depths()).to(dev)
    st = torch.cuda.current_stream(dev)

    def device_step():
        eng.step(ids_d, par_d, dep_d, 0, PROMPT)

    # correctness of the timed configuration: the AR chain is accepted in full
    am = eng.verify(tree, PROMPT, 0)
    path, acc, rec = walk(tree, first, 1 << 30, -1, lambda a, ch: int(am[ch]))
    committed = len(acc)
    assert acc == toks[:chain_n] and committed == chain_n, "trie verify disagrees with AR decoding"

    for _ in range(args.warmup):
        device_step()
    torch.cuda.synchronize()

    def timed(fn, k):
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        for _ in range(k):
            fn()
        e1.record(st)
        torch.cuda.synchronize()
        return reduce_max(e0.elapsed_time(e1), dev)

    with Clocks(local) as clk:
        ms = timed(device_step, args.steps)
    clocks = clk.summary()
    ms_step = ms / args.steps
    value = job_value(world, committed, args.steps, ms)

    # e2e: the public calls with host trie arrays (copied in), the acceptance walk and
    # KV compaction on the device, and the acceptance record read back to the host
    h_ids, h_par, h_dep = tree.tokens().astype(np.int32), tree.parents(), tree.depths()

    def e2e_step():
        eng.step(h_ids, h_par, h_dep, 0, PROMPT)
        p, a, r = eng.accept(first, 1 << 30, -1, n=NODES)
        assert len(a) == committed

    k2 = args.e2e_steps or max(1, args.steps // 3)
    for _ in range(2):
        e2e_step()
    ms2 = timed(e2e_step, k2)
    e2e = {"value": job_value(world, committed, k2, ms2), "unit": "committed tokens/s",
           "ms_per_step": ms2 / k2, "h2d_bytes_per_step": 32 + 3 * 4 * NODES, "d2h_bytes_per_step": 4 * (4 + 2 * NODES),
           "path": "VerifyEngine.step (host trie arrays) + VerifyEngine.accept (device walk + KV compaction)"}

    # roofline of the dominant kernel: the fused gate|up + SiLU*mul GEMM of a layer
    hbm, tf, src = measured_peaks()
    xg = torch.randn(NODES, cfg.hidden, device=dev, generator=torch.Generator(device=dev).manual_seed(5)).to(torch.bfloat16)
    ngu = 2 * cfg.ffn
    bufs = [pk["wgu"] for pk in eng.packed]   # the engine's packed gate|up weights, one per layer
    for _ in range(3):
        linear_swiglu_packed(xg, bufs[0], cfg.ffn)
    reps = 56
    # captured in a CUDA graph so that host launch overhead does not enter the timing;
    # layers rotate so every launch streams its weights from HBM
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for i in range(reps):
            linear_swiglu_packed(xg, bufs[i % len(bufs)], cfg.ffn)
    g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    g.replay()
    e1.record(st)
    torch.cuda.synchronize()
    gu_ms = e0.elapsed_time(e1) / reps
    gu_bytes = ngu * cfg.hidden * 2 + xg.numel() * 2 + NODES * cfg.ffn * 2
    achieved = gu_bytes / (gu_ms * 1e-3) / 1e9
    step_bytes = cfg.weight_bytes_per_step() + 2 * cfg.n_layers * 2 * cfg.n_kv_heads * (PROMPT + NODES) * 128 \
        + NODES * cfg.vocab * 4
    roof = {"bound": "hbm", "kernel": "gemm_kernel<256,1,kEpiSiluMul> fused gate|up+SiLU*mul N=37888 K=3584 M=128",
            "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm, "peak_source": src,
            "traffic": profiled_traffic(),
            "traffic_source": "committed ncu capture of this kernel (profiles/gemm_gate_up_config3.md), "
                              "not a per-run measurement",
            "algorithmic_bytes": gu_bytes, "launch_ms": gu_ms}
    step_roof = {"bound": "hbm", "algorithmic_bytes": step_bytes, "achieved": step_bytes / (ms_step * 1e-3) / 1e9,
                 "peak": hbm, "unit": "GB/s", "frac": step_bytes / (ms_step * 1e-3) / 1e9 / hbm,
                 "floor_ms": step_bytes / (hbm * 1e9) * 1e3}

    # config 5 beside it: the multi-stream frame replay on this GPU (weights shared with
    # the config-3 engine), so every run, the scaling runs included, records frames/s
    replay = None
    if args.replay_frames > 0:
        r = replay_measure(w, world, rank, local, dev, args.replay_streams, 1, args.replay_frames, share=eng)
        st = r["stats"]
        replay = {"metric": "frames/s (multi-stream frame replay, config 5)", "value": r["value"],
                  "unit": "frames/s", "n_gpus": world, "scaling": "weak", "streams_per_gpu": args.replay_streams,
                  "warmup_frames_per_stream": 1, "frames_per_stream": args.replay_frames, "ms": r["ms"],
                  "frames": r["frames"], "rounds": st.rounds, "prefill_steps": st.prefill_steps,
                  "tokens_per_round": st.tokens_per_round(), "ms_per_step": r["ms"] / max(r["n_steps"], 1),
                  "floor_frac": r["roofline"]["frac"], "step_floor_ms": r["roofline"]["step_floor_ms"],
                  "bound": r["roofline"]["bound"], "clocks": r["clocks"],
                  "workload": "16 frame streams per GPU, 4096-token prompts 90% shared with the previous frame, "
                              "256-node tries, 80 committed tokens per frame; one untimed frame per stream, "
                              "then the timed frames, max over ranks"}
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cb = cpu_steps(2, 1, nodes=NODES, prompt=PROMPT)
        cpu = {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")}
    err = _lib.device_error()
    launches = args.steps * (KERNELS_FIXED + KERNELS_PER_LAYER * cfg.n_layers)
    if rank == 0:
        line = {"metric": "committed tokens/s (trie-verify step)", "value": value, "unit": "committed tokens/s",
                "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
                "data": "synthetic (seeded ids, random-init weights)", "config": config_block(world, NODES, PROMPT),
                "e2e": e2e, "gpu_launches": launches, "roofline": roof, "step_roofline": step_roof,
                "cpu_baseline": cpu, "clocks": clocks, "frame_replay": replay, "device_error": err}
        print(json.dumps(line), flush=True)
    eng.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


# ------------------------------------------------------------------ frame replay
def replay_measure(w, world, rank, local, dev, streams, warm_frames, frames_per_stream, one_cuda_stream=False,
                   share=None):
    """The config-5 frame replay on this rank's GPU: `streams` frame streams (one
    VerifyEngine each on shared weights; `share`: an engine of the same weights whose
    packed copy they reuse), `warm_frames` untimed frames per stream, then
    `frames_per_stream` timed ones between CUDA events (all ranks start together;
    the max over ranks is taken). Returns the measurement and its floor."""
    import torch.distributed as dist

    from respect_b200.decoding.engine import VerifyEngine
    from respect_b200.decoding.replay import FrameReplay, ReplayConfig
    cfg = w.cfg
    rcfg = ReplayConfig(streams=streams, seed=1000 + rank, shared_cuda_stream=one_cuda_stream)
    engines = None
    if share is not None:
        rows = max(rcfg.trie_nodes, rcfg.prefill_chunk)
        engines = [VerifyEngine(w, max_rows=rows, max_slots=rcfg.max_slots(), share_weights=share)
                   for _ in range(streams)]
    rep = FrameReplay(w, rcfg, engines=engines)
    warm = rep.run(warm_frames)
    if world > 1:
        dist.barrier()
    with Clocks(local) as clk:
        stats, ms = rep.timed_run(frames_per_stream)
    ms = reduce_max(ms, dev)
    clocks = clk.summary()
    frames = stats.frames
    value = world * frames / (ms / 1e3)
    # floor of the steps the timed frames ran (prefill chunks and verification
    # rounds, 256 rows each): max(HBM bytes / peak, tensor FLOPs / peak) per step
    hbm, tf, src = measured_peaks()
    rows = rcfg.trie_nodes
    keys = rcfg.prompt_len + rcfg.commit_tokens // 2 + rows // 2
    kv_bytes = 2 * cfg.n_layers * 2 * cfg.n_kv_heads * keys * cfg.head_dim
    step_bytes = cfg.weight_bytes_per_step() + kv_bytes + rows * cfg.vocab * 4
    mm_flops = 2 * rows * (cfg.n_layers * cfg.layer_params() + cfg.vocab * cfg.hidden)
    attn_flops = 4 * rows * cfg.n_layers * cfg.n_heads * cfg.head_dim * keys
    t_hbm_ms = step_bytes / (hbm * 1e9) * 1e3
    t_tc_ms = (mm_flops + attn_flops) / (tf * 1e12) * 1e3
    n_steps = stats.rounds + stats.prefill_steps
    floor_ms = n_steps * max(t_hbm_ms, t_tc_ms)
    roof = {"bound": "hbm" if t_hbm_ms >= t_tc_ms else "tensor", "step_floor_ms": max(t_hbm_ms, t_tc_ms),
            "unit": "ms", "floor_ms": floor_ms, "achieved_ms": ms, "frac": floor_ms / ms,
            "peak_hbm_gbs": hbm, "peak_tflops": tf, "peak_source": src,
            "step_bytes": step_bytes, "step_flops": mm_flops + attn_flops, "steps": n_steps,
            "traffic": None}
    per_round = 32 + 3 * 4 * rows
    h2d = (stats.prefill_tokens * 12 + stats.prefill_steps * 32 + stats.rounds * per_round) / max(frames, 1)
    d2h = (stats.rounds * 4 * (4 + 2 * rows) + frames * 8 * rcfg.prefill_chunk) / max(frames, 1)
    rep.close()
    return dict(rcfg=rcfg, stats=stats, warm=warm, ms=ms, value=value, clocks=clocks, frames=frames, rows=rows,
                n_steps=n_steps, roofline=roof, h2d=h2d, d2h=d2h)


def run_frame_replay(args):
    """Multi-stream frame replay: --streams frame streams per GPU (16 by default),
    each frame a 4,096-token prompt (90% shared with the previous frame, Prefill
    reusing the unchanged chunks) and 256-node verification rounds until 80 tokens
    are committed. --warmup frames per stream untimed, then --steps frames per
    stream timed. Metric: frames/s (whole job)."""
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=900), device_id=dev)

    from respect_b200 import _lib
    from respect_b200.decoding.engine import DecoderConfig, DecoderWeights

    cfg = DecoderConfig.baseline_7b()
    w = DecoderWeights.random(cfg, dev, seed=0)
    r = replay_measure(w, world, rank, local, dev, args.streams, args.warmup, args.steps, args.one_cuda_stream)
    rcfg, stats, ms, value, clocks = r["rcfg"], r["stats"], r["ms"], r["value"], r["clocks"]
    frames, rows, n_steps, roof, h2d, d2h = r["frames"], r["rows"], r["n_steps"], r["roofline"], r["h2d"], r["d2h"]
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        # whole 256-row steps of the reference's eager path at the 4096-token prefix,
        # times the steps the timed frames ran (prefill chunks counted as full-prefix
        # steps: an upper bound)
        cb = cpu_steps(2, 1, nodes=rows, prompt=rcfg.prompt_len, chain=rcfg.chain_len)
        cpu_frame_s = n_steps * cb["ms_per_step"] / 1e3 / max(frames, 1)
        cpu = {"value": 1.0 / cpu_frame_s, "unit": "frames/s", "cores": cb["cores"], "kind": "port",
               "sample": cb["sample"] + f"; a frame = {n_steps / max(frames, 1):.1f} such steps (the timed "
                         f"frames' prefill chunks and rounds) = {cpu_frame_s:.0f} s"}
    err = _lib.device_error()
    if rank == 0:
        line = {"metric": "frames/s (multi-stream frame replay)", "value": value, "unit": "frames/s",
                "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                "dtype": "bf16", "data": "synthetic (seeded prompts and edits, random-init weights)",
                "config": {"workload": "frame replay: 28-layer 7B-class decoder, 4096-token prompts 90% shared "
                                       "with the previous frame, 256-node tries (4 chains of 48 + continuation "
                                       "nodes), 80 committed tokens per frame",
                           "streams_per_gpu": rcfg.streams, "frames_per_stream": args.steps,
                           "cuda_streams": 1 if rcfg.shared_cuda_stream else rcfg.streams,
                           "parallelism": f"replicas{world}",
                           "l2": "inputs larger than L2 (14.1 GB weights per step)"},
                "e2e": {"value": value, "unit": "frames/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                        "path": "FrameReplay.run: host prompts -> VerifyEngine.prefill, host tries -> "
                                "VerifyEngine.step, device acceptance record -> host; the timed region is "
                                "end to end (bytes per frame)"},
                "gpu_launches": n_steps * (KERNELS_FIXED + KERNELS_PER_LAYER * cfg.n_layers) + stats.rounds * 2,
                "roofline": roof, "cpu_baseline": cpu,
                "replay": {"frames": frames, "rounds": stats.rounds, "committed": stats.committed,
                           "tokens_per_round": stats.tokens_per_round(), "prefill_steps": stats.prefill_steps,
                           "prefill_tokens_per_frame": stats.prefill_tokens / max(frames, 1),
                           "warmup_frames": r["warm"].frames},
                "clocks": clocks, "device_error": err}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


# ------------------------------------------------------------------ single-kernel cases
def _median_launch_us(torch, fn, reps, flush, inner=20):
    """Device time of one fn() launch that follows an L2 flush (a write of a buffer
    larger than L2), net of the flush: two CUDA graphs, `inner` x (flush, fn) and
    `inner` x (flush), each replayed between CUDA events; the median over `reps`
    replays of their difference, divided by `inner`. One graph launch per `inner`
    operations keeps the host and the launch latency out of the figure."""
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        fn()
    torch.cuda.current_stream().wait_stream(side)
    g_op, g_fl = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
    with torch.cuda.graph(g_op):
        for _ in range(inner):
            flush.zero_()
            fn()
    with torch.cuda.graph(g_fl):
        for _ in range(inner):
            flush.zero_()

    def timed(g):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        g.replay()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) * 1e3

    g_op.replay()
    g_fl.replay()
    torch.cuda.synchronize()
    diffs = [(timed(g_op) - timed(g_fl)) / inner for _ in range(max(reps // inner, 5))]
    return statistics.median(diffs)


def _median_cpu_ms(fn, reps):
    ts = []
    for _ in range(reps):
        t0 = time.perf_counter()
        fn()
        ts.append((time.perf_counter() - t0) * 1e3)
    return statistics.median(ts)


def run_config_case(args):
    """Configs 1 and 2: the standalone operators at their BASELINE shapes, timed per
    launch after an L2 flush (their inputs fit in L2), next to PyTorch eager on the
    host cores at the same shapes (the reference's CPU path for these operators)."""
    import torch
    dev = torch.device("cuda", 0)
    hbm, _, src = measured_peaks()
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    reps, warm = max(args.steps, 20), max(args.warmup, 3)
    threads = torch.get_num_threads()
    lines = []
    if args.kernel_case == "config1":
        from oracle.inputs import attention_case
        from respect_b200.kernels.attention import fused_attn_hyb
        c = attention_case(0)
        t = {k: torch.from_numpy(np.ascontiguousarray(c[k])) for k in ("q", "kp", "vp", "kn", "vn", "msk")}
        g = {k: v.to(dev) for k, v in t.items()}
        fn = lambda: fused_attn_hyb(g["q"], g["kp"], g["vp"], g["kn"], g["vn"], g["msk"])  # noqa: E731
        for _ in range(warm):
            fn()
        us = _median_launch_us(torch, fn, reps, flush)
        H, M, D = c["q"].shape
        HK, NP, _ = c["kp"].shape
        NN = c["kn"].shape[1]
        algo = 4 * (2 * HK * (NP + NN) * D + 2 * H * M * D) + M * NN
        # eager SDPA on the CPU (dispatch's original path): fp32, additive mask over [prefix | nodes]
        G = H // HK
        qc = t["q"][None]
        kc = torch.cat([t["kp"], t["kn"]], 1).repeat_interleave(G, 0)[None]
        vc = torch.cat([t["vp"], t["vn"]], 1).repeat_interleave(G, 0)[None]
        mask = torch.zeros(M, NP + NN)
        mask[:, NP:] = torch.where(t["msk"], 0.0, float("-inf"))
        cpu = lambda: torch.nn.functional.scaled_dot_product_attention(qc, kc, vc, attn_mask=mask)  # noqa: E731
        cpu()
        cpu_ms = _median_cpu_ms(cpu, 20)
        lines.append({"op": "fused_attn_hyb fp32 (config 1)", "shape": f"H{H}/{HK} M{M} NP{NP} NN{NN} D{D}",
                      "us": us, "algorithmic_bytes": algo})
        lines[-1]["cpu_ms"] = cpu_ms
    else:
        from respect_b200.kernels.rmsnorm import rmsnorm
        from respect_b200.system.fused import rope, silu_mul
        gen = torch.Generator().manual_seed(0)
        x = torch.randn(128, 3584, generator=gen).to(torch.bfloat16)
        w = (torch.rand(3584, generator=gen) + 0.5).to(torch.bfloat16)
        rng = np.random.default_rng(0)
        parents = [-1] + [int(rng.integers(0, i)) for i in range(1, 128)]
        depth = [0] * 128
        for i in range(1, 128):
            depth[i] = depth[parents[i]] + 1
        pos = torch.tensor([3000 + d for d in depth], dtype=torch.float32)
        inv = 1.0 / (1e6 ** (torch.arange(0, 128, 2, dtype=torch.float32) / 128))
        f = pos[:, None] * inv[None]
        emb = torch.cat([f, f], -1)
        cos, sin = emb.cos().to(torch.bfloat16)[None], emb.sin().to(torch.bfloat16)[None]
        q = torch.randn(1, 28, 128, 128, generator=gen).to(torch.bfloat16)
        k = torch.randn(1, 4, 128, 128, generator=gen).to(torch.bfloat16)
        gt = torch.randn(128, 18944, generator=gen).to(torch.bfloat16)
        ut = torch.randn(128, 18944, generator=gen).to(torch.bfloat16)
        xd, wd, cd, sd, qd, kd, gd, ud = (v.to(dev) for v in (x, w, cos, sin, q, k, gt, ut))

        def rot(v):
            return torch.cat([-v[..., 64:], v[..., :64]], -1)

        def hf_norm(v, wt):
            vf = v.float()
            return wt * (vf * torch.rsqrt(vf.pow(2).mean(-1, keepdim=True) + 1e-6)).to(v.dtype)
        ops = [("rmsnorm (row-invariant) [128, 3584]", lambda: rmsnorm(xd, wd, 1e-6), lambda: hf_norm(x, w),
                3 * 128 * 3584 * 2 + 3584 * 2),
               ("rope q [1,28,128,128] + k [1,4,128,128]", lambda: (rope(qd, cd, sd), rope(kd, cd, sd)),
                lambda: (q * cos[:, None] + rot(q) * sin[:, None], k * cos[:, None] + rot(k) * sin[:, None]),
                2 * 2 * (28 + 4) * 128 * 128 + 2 * 2 * 128 * 128 * 2),
               ("silu_mul [128, 18944]", lambda: silu_mul(gd, ud),
                lambda: torch.nn.functional.silu(gt) * ut, 3 * 128 * 18944 * 2)]
        for name, gpu_fn, cpu_fn, algo in ops:
            for _ in range(warm):
                gpu_fn()
            us = _median_launch_us(torch, gpu_fn, reps, flush)
            cpu_fn()
            lines.append({"op": name, "us": us, "algorithmic_bytes": algo, "cpu_ms": _median_cpu_ms(cpu_fn, 20)})
    for ln in lines:
        ln.update({"kernel_case": args.kernel_case, "GBps": ln["algorithmic_bytes"] / (ln["us"] * 1e-6) / 1e9,
                   "peak_hbm_gbs": hbm, "peak_source": src, "cpu_threads": threads,
                   "cpu_over_gpu": ln["cpu_ms"] * 1e3 / ln["us"],
                   "l2": "flushed before every launch; the flush's own time subtracted",
                   "launches": reps})
        ln["frac"] = ln["GBps"] / hbm
        print(json.dumps(ln), flush=True)


def run_kernel_case(args):
    import torch
    from respect_b200.decoding.engine import DecoderConfig
    dev = torch.device("cuda", 0)
    cfg = DecoderConfig.baseline_7b()
    NODES, PROMPT = args.nodes, args.prefix  # noqa: N806 (config 3: 128, 3000)
    g = torch.Generator(device=dev).manual_seed(7)
    st = torch.cuda.current_stream(dev)
    if args.kernel_case == "step_small":
        from oracle.inputs import chain_seqs, top_up
        from respect_b200.candidates.trie import build_trie
        from respect_b200.decoding.engine import DecoderWeights, VerifyEngine
        c1 = DecoderConfig(cfg.hidden, 1, cfg.n_heads, cfg.n_kv_heads, cfg.head_dim, cfg.ffn, cfg.vocab)
        w = DecoderWeights.random(c1, dev, seed=0)
        eng = VerifyEngine(w, max_rows=NODES, max_slots=PROMPT + 1024)
        rng = np.random.default_rng(100)
        eng.prefill(rng.integers(0, c1.vocab, PROMPT))
        tree = build_trie(top_up(rng, chain_seqs(rng, 4, 32, c1.vocab), NODES, c1.vocab))
        ids_d = torch.from_numpy(tree.tokens().astype(np.int32)).to(dev)
        par_d = torch.from_numpy(tree.parents()).to(dev)
        dep_d = torch.from_numpy(tree.depths()).to(dev)

        def launch(i):
            eng.step(ids_d, par_d, dep_d, 0, PROMPT)
        algo = c1.weight_bytes_per_step()
        flops = 2 * NODES * (c1.layer_params() + c1.vocab * c1.hidden)
    elif args.kernel_case == "gemm_gate_up":
        from respect_b200.kernels.gemm import linear_swiglu_packed, pack_gate_up
        h, F = cfg.hidden, cfg.ffn
        ws = []
        for _ in range(2):
            wg = (torch.randn(F, h, device=dev, generator=g) * 0.02).to(torch.bfloat16)
            wu = (torch.randn(F, h, device=dev, generator=g) * 0.02).to(torch.bfloat16)
            ws.append(pack_gate_up(wg, wu))
            del wg, wu
        x = torch.randn(NODES, h, device=dev, generator=g).to(torch.bfloat16)

        def launch(i):
            linear_swiglu_packed(x, ws[i % 2], F)
        algo = 2 * F * h * 2 + NODES * h * 2 + NODES * F * 2
        flops = 2 * NODES * 2 * F * h
    else:
        from respect_b200.kernels.attention import fused_attn_hyb
        from oracle.trie import ancestry
        H, HK, D = cfg.n_heads, cfg.n_kv_heads, cfg.head_dim
        q = (torch.randn(H, NODES, D, device=dev, generator=g) / D ** 0.5).to(torch.bfloat16)
        kc = torch.randn(HK, PROMPT + 1024, D, device=dev, generator=g).to(torch.bfloat16)
        vc = torch.randn(HK, PROMPT + 1024, D, device=dev, generator=g).to(torch.bfloat16)
        rng = np.random.default_rng(3)
        parents = [-1] + [int(rng.integers(0, i)) for i in range(1, NODES)]
        msk = torch.from_numpy(ancestry(parents)).to(dev)
        kp, vp = kc[:, :PROMPT], vc[:, :PROMPT]
        kn, vn = kc[:, PROMPT:PROMPT + NODES], vc[:, PROMPT:PROMPT + NODES]

        def launch(i):
            fused_attn_hyb(q, kp, vp, kn, vn, msk)
        algo = 2 * HK * (PROMPT + NODES) * D * 2 + 2 * H * NODES * D * 2
        flops = 4 * H * NODES * PROMPT * D
    for i in range(args.warmup):
        launch(i)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for i in range(args.steps):
        launch(i)
    e1.record(st)
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / args.steps
    print(json.dumps({"kernel_case": args.kernel_case, "launches": args.steps, "us_per_launch": us,
                      "rows": NODES, "algorithmic_bytes": algo, "GBps": algo / (us * 1e-6) / 1e9,
                      "tensor_flops": flops, "TFLOPs": flops / (us * 1e-6) / 1e12}), flush=True)


def main():
    args = parse()
    if args.kernel_case in ("config1", "config2"):
        run_config_case(args)
    elif args.kernel_case:
        run_kernel_case(args)
    elif args.impl == "reference":
        run_reference(args)
    elif args.workload == "frame_replay":
        run_frame_replay(args)
    else:
        run_native(args)


if __name__ == "__main__":
    main()
