"""Benchmark of the SISA hot path on B200 (one JSON line on rank 0).

Workload: SISA attention forward + backward including the fused preparation,
B=8, T=4096, H=16, d_head 64, d_state 32, bf16 operands with fp32 g/F, from a fused projection
``proj`` (B, T, NPAD) and forget logits ``z``. One step = sisa_prep_fwd, sisa_attn_fwd, sisa_attn_bwd,
sisa_prep_bwd through the C ABI (the same calls the autograd wrapper makes), on buffers allocated
once. Metric: TFLOP/s on the causal FLOP count, 1152 FLOP per causal (query, key) pair
(fwd 2(2*64+32), bwd 2(5*64+3*32)). With N ranks each rank runs its own batch (weak scaling, no
collective on the data path); ``value`` = all ranks' FLOPs / max-over-ranks time.

``e2e``: the same step with host buffers: pinned proj/z/dy copied in, y/d_proj/dz/dlam copied out,
every step, inside the timed region; copies and compute of consecutive steps overlap (two device
buffer sets, separate copy streams).

``train``: the second half of the metric, 12-layer sisa-152m training (d=768, H=12, d_ff=2744, vocab
50277, reference initialisation) with per-rank batch 8 x 2048 uniform random ids, bf16 autocast, fused
AdamW, clipping, fused linear-CE, data-parallel over the N ranks: the whole step is one CUDA graph per
rank, and the fp32 gradients are averaged by NCCL allreduces of buckets issued on a second captured
stream as the backward finishes each bucket (sisa_b200/dp.py). tokens/s = all ranks' input tokens /
max-over-ranks step time.

On one GPU the default run also reports BASELINE config 2 (``lce``: chunked linear-CE fwd+bwd) and
config 4 (``decode``: prefill and graphed decode steps of the 12-layer model), and ``incumbent``: the
reference's own Triton ``sisa_fused`` (installed under baseline/_ref) on the same cfg1 inputs, each with
the reference's GPU number beside it where the reference has that path.

``--impl reference``: the reference's pure-PyTorch CPU algorithm (the oracle port) on the host cores,
on a bounded sample of the same workload (a subset of (batch, head) units at the full T).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

B, T, H = 8, 4096, 16
FLOP_PER_PAIR = 1152
FWD_FLOP_PER_PAIR = 320
# DRAM bytes (read + write) of attn_fwd + attn_bwd_dq + attn_bwd_dkv for one cfg1 step: ncu
# dram__bytes_read.sum + dram__bytes_write.sum of one capture at B=1, H=8, T=4096, scaled by the number
# of (batch, head, position) units; the traffic per unit does not depend on B or H.
ATTN_TRAFFIC_PER_UNIT = 1.1537e9 / (8 * 16 * 4096)
METRIC = "SISA attn fwd+bwd TFLOP/s (T=4096 bf16)"


def pairs(b, h, t):
    return b * h * t * (t + 1) // 2


def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d.get("bf16_tflops", 1590.0), d.get("bf16_tflops_sustained", 1400.0), d.get("hbm_gbs", 6650.0), "measured"
    return 1590.0, 1400.0, 6650.0, "fallback"


class Clocks:
    """Samples the SM clock and the clock-event (throttle) reasons of one GPU through NVML every
    ``period`` seconds on a background thread, from ``start()`` to ``stop()``. ``window(name)`` marks a
    region (the timed steps); ``summary(name)`` reports the samples inside it."""

    REASONS = (("hw_slowdown", "nvmlClocksEventReasonHwSlowdown"),
               ("hw_thermal_slowdown", "nvmlClocksEventReasonHwThermalSlowdown"),
               ("sw_thermal_slowdown", "nvmlClocksEventReasonSwThermalSlowdown"),
               ("hw_power_brake_slowdown", "nvmlClocksEventReasonHwPowerBrakeSlowdown"),
               ("sw_power_cap", "nvmlClocksEventReasonSwPowerCap"))

    def __init__(self, device_index, period=0.004):
        self.period = period
        self.samples = []          # (host time, sm MHz, reason bits)
        self.windows = {}
        self.max_mhz = None
        self._stop = None
        self._thread = None
        self._nvml = None
        self._handle = None
        try:
            import pynvml

            pynvml.nvmlInit()
            handle = None
            try:
                uuid = str(torch.cuda.get_device_properties(device_index).uuid)
                handle = pynvml.nvmlDeviceGetHandleByUUID(uuid if uuid.startswith("GPU-") else "GPU-" + uuid)
            except Exception:  # noqa: BLE001
                handle = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self._nvml, self._handle = pynvml, handle
            self.max_mhz = float(pynvml.nvmlDeviceGetMaxClockInfo(handle, pynvml.NVML_CLOCK_SM))
        except Exception:  # noqa: BLE001
            self._nvml = None

    def _run(self):
        nv, h = self._nvml, self._handle
        while not self._stop.is_set():
            try:
                mhz = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
                bits = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
                self.samples.append((time.perf_counter(), float(mhz), int(bits)))
            except Exception:  # noqa: BLE001
                pass
            self._stop.wait(self.period)

    def start(self):
        if self._nvml is not None and self._thread is None:
            import threading

            self._stop = threading.Event()
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        return self

    def stop(self):
        if self._thread is not None:
            self._stop.set()
            self._thread.join(timeout=5)
            self._thread = None

    def __enter__(self):
        return self.start()

    def __exit__(self, *a):
        self.stop()

    def window(self, name):
        clk = self

        class _W:
            def __enter__(self):
                clk.windows[name] = [time.perf_counter(), None]

            def __exit__(self, *a):
                clk.windows[name][1] = time.perf_counter()
        return _W()

    def summary(self, name=None):
        if self._nvml is None:
            return None
        rows = self.samples
        if name is not None and name in self.windows and self.windows[name][1] is not None:
            t0, t1 = self.windows[name]
            rows = [r for r in rows if t0 <= r[0] <= t1]
        if not rows:
            return None
        reasons = sorted({label for _, _, bits in rows for label, const in self.REASONS
                          if bits & getattr(self._nvml, const, 0)})
        return {"sm_mhz": statistics.median(r[1] for r in rows), "sm_max_mhz": self.max_mhz, "reasons": reasons,
                "samples": len(rows), "window": name or "whole run", "source": f"NVML every {self.period * 1e3:.0f} ms"}


def dist_setup(n):
    if n <= 1 or int(os.environ.get("WORLD_SIZE", "1")) <= 1:
        return 0, 1, 0
    import datetime

    import torch.distributed as dist

    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    return dist.get_rank(), dist.get_world_size(), local


class Step:
    """Buffers and the four C-ABI calls of one fused-layer forward + backward."""

    def __init__(self, dev, b=B, t=T, h=H, seed=0):
        from sisa_b200 import _lib, backends
        from sisa_b200.kernels.fused import fused_layout

        self.lib = _lib.load()
        self._lib = _lib
        self.dev, self.b, self.t, self.h = dev, b, t, h
        off = fused_layout(h)
        self.off = off
        g = torch.Generator(device=dev).manual_seed(seed)
        bf = dict(device=dev, dtype=torch.bfloat16)
        f32 = dict(device=dev, dtype=torch.float32)
        proj = torch.zeros((b, t, off["NPAD"]), **bf)
        proj[..., :off["TH"]] = torch.randn((b, t, off["TH"]), generator=g, device=dev).to(torch.bfloat16)
        proj[..., off["TH"]:off["A"]] = (torch.randn((b, t, h * 16), generator=g, device=dev) * 0.2).to(torch.bfloat16)
        proj[..., off["A"]:off["NTOT"]] = (torch.randn((b, t, h), generator=g, device=dev) * 0.45 - 5).to(torch.bfloat16)
        self.proj = proj
        self.z = torch.randn((b, t, h), generator=g, device=dev) * 0.45 + 4
        self.lam = torch.nn.functional.softplus(torch.full((h,), -1.0, **f32))
        self.dy = torch.randn((b, t, h * 64), generator=g, device=dev).to(torch.bfloat16)
        self.c_rot = torch.empty((b, h, t, 32), **bf)
        self.b_rot = torch.empty((b, h, t, 32), **bf)
        self.pos = _lib.pos_planes(b, h, t, dev)
        self.tot = torch.empty(self.lib.sisa_prep_fwd_workspace(b, h, t), dtype=torch.uint8, device=dev)
        self.o = torch.empty_strided((b, h, t, 64), (t * h * 64, 64, h * 64, 1), **bf)
        self.lse = torch.empty((b, h, t), **f32)
        self.o32 = torch.empty((b, h, t, 64), **f32)
        self.dproj = torch.empty_like(proj)
        self.dc = torch.empty((b, h, t, 32), **f32)
        self.db = torch.empty((b, h, t, 32), **f32)
        self.dg = torch.empty((b, h, t), **f32)
        self.dF = torch.empty((b, h, t), **f32)
        self.dlam = torch.empty((h,), **f32)
        self.dz = torch.empty((b, t, h), **f32)
        self.ws = torch.empty(self.lib.sisa_attn_bwd_workspace(b, h, t), dtype=torch.uint8, device=dev)
        self.bt = torch.empty(self.lib.sisa_prep_bwd_workspace(b, h, t), dtype=torch.uint8, device=dev)
        self.status = backends.status_word(dev)
        heads = lambda x, c, w: x[..., c:c + h * w].view(b, t, h, w).transpose(1, 2)  # noqa: E731
        do = self.dy.view(b, t, h, 64).transpose(1, 2)
        tens = [heads(proj, off["Q"], 64), heads(proj, off["K"], 64), heads(proj, off["V"], 64), self.c_rot,
                self.b_rot, self.o, do, heads(self.dproj, off["Q"], 64), heads(self.dproj, off["K"], 64),
                heads(self.dproj, off["V"], 64), self.dc, self.db]
        self.views = [_lib.view4(x) for x in tens]
        self.refs = [_lib.vref(v) for v in self.views]
        self.launches_per_step = 8   # prep: 2, attn fwd: 1, attn bwd: 3 (dq, dkv, dlam), prep bwd: 2

    def prep_fwd(self, st):
        L = self.lib
        rc = L.sisa_prep_fwd(self.proj.data_ptr(), self.b, self.t, self.h, self.proj.stride(0), self.proj.stride(1),
                             0, self.z.data_ptr(), self.z.stride(0), self.z.stride(1), self.c_rot.data_ptr(),
                             self.b_rot.data_ptr(), self.pos.data_ptr(), self.tot.data_ptr(), self.status.data_ptr(), st)
        self._lib.check(rc, "sisa_prep_fwd")

    def attn_fwd(self, st):
        r = self.refs
        rc = self.lib.sisa_attn_fwd(r[0], r[1], r[2], r[3], r[4], self.pos.data_ptr(), self.lam.data_ptr(), self.b,
                                    self.h, self.t, 0, r[5], self.lse.data_ptr(), self.o32.data_ptr(),
                                    self.status.data_ptr(), st)
        self._lib.check(rc, "sisa_attn_fwd")

    def attn_bwd(self, st):
        r = self.refs
        rc = self.lib.sisa_attn_bwd(r[0], r[1], r[2], r[3], r[4], self.pos.data_ptr(), self.lam.data_ptr(), r[5],
                                    r[6], self.lse.data_ptr(), self.o32.data_ptr(), self.b, self.h, self.t, 0, r[7],
                                    r[8], r[9], r[10], r[11], self.dg.data_ptr(), self.dF.data_ptr(),
                                    self.dlam.data_ptr(), self.ws.data_ptr(), self.status.data_ptr(), st)
        self._lib.check(rc, "sisa_attn_bwd")

    def prep_bwd(self, st):
        rc = self.lib.sisa_prep_bwd(self.proj.data_ptr(), self.b, self.t, self.h, self.proj.stride(0),
                                    self.proj.stride(1), 0, self.z.data_ptr(), self.z.stride(0), self.z.stride(1),
                                    self.tot.data_ptr(), self.dc.data_ptr(), self.db.data_ptr(), self.dg.data_ptr(),
                                    self.dF.data_ptr(), self.dproj.data_ptr(), self.dproj.stride(0),
                                    self.dproj.stride(1), self.dz.data_ptr(), self.bt.data_ptr(),
                                    self.status.data_ptr(), st)
        self._lib.check(rc, "sisa_prep_bwd")

    def run(self, st, ev=None):
        if ev is None:
            self.prep_fwd(st); self.attn_fwd(st); self.attn_bwd(st); self.prep_bwd(st)  # noqa: E702
            return
        ev[0].record(); self.prep_fwd(st)  # noqa: E702
        ev[1].record(); self.attn_fwd(st)  # noqa: E702
        ev[2].record(); self.attn_bwd(st)  # noqa: E702
        ev[3].record(); self.prep_bwd(st)  # noqa: E702
        ev[4].record()


def run_cuda(args):
    rank, world, local = dist_setup(args.gpus)
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    from sisa_b200 import backends

    ok, why = backends.cuda_status(local)
    if not ok:
        raise RuntimeError(f"cuda kernels unavailable: {why}")
    step = Step(dev, b=args.B, t=args.T, h=args.H, seed=1234 + rank)
    stream = torch.cuda.current_stream(dev)
    st = stream.cuda_stream
    clk = Clocks(local).start()          # sampled through the whole run; the timed steps are a window
    for _ in range(args.warmup):
        step.run(st)
    torch.cuda.synchronize(dev)
    backends.check_status(dev)
    # ---- timed region: K steps, per-call events on the launching stream
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(5)] for _ in range(args.steps)]
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize(dev)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with clk.window("timed"):
        start.record()
        for k in range(args.steps):
            step.run(st, evs[k])
        end.record()
        torch.cuda.synchronize(dev)
    if world > 1:
        torch.distributed.barrier()
    ms = start.elapsed_time(end)
    per = {name: statistics.mean(e[i].elapsed_time(e[i + 1]) for e in evs)
           for i, name in enumerate(["prep_fwd", "attn_fwd", "attn_bwd", "prep_bwd"])}
    backends.check_status(dev)
    ms_t = torch.tensor([ms], device=dev)
    if world > 1:
        torch.distributed.all_reduce(ms_t, op=torch.distributed.ReduceOp.MAX)
    ms_max = float(ms_t.item())
    b_, t_, h_ = args.B, args.T, args.H
    total_flop = FLOP_PER_PAIR * pairs(b_, h_, t_) * args.steps * world
    value = total_flop / (ms_max * 1e-3) / 1e12

    # ---- e2e: host buffers in and out through the same C-ABI calls
    e2e = None if args.no_e2e else run_e2e(step, dev, args, world)
    proj_mb = step.proj.numel() * 2 / 1e6
    inputs = (step.proj, step.z, step.lam, step.dy)
    del step
    torch.cuda.empty_cache()
    # BASELINE configs 2 and 4 and the reference's own GPU path, on one GPU only (replicas add nothing)
    extra = {}
    if world == 1 and not args.no_extra:
        extra["incumbent"] = incumbent_leg(inputs, args)
        del inputs
        torch.cuda.empty_cache()
        extra["lce"] = lce_leg(args, dev)
        torch.cuda.empty_cache()
        extra["decode"] = decode_leg(args, dev, steps=args.extra_decode_steps)
        torch.cuda.empty_cache()
        extra["gemm"] = gemm_leg(args, dev, n=args.gemm_size, steps=10)
        torch.cuda.empty_cache()
    else:
        del inputs
    with clk.window("train"):
        train = None if args.no_train else run_train(args, rank, world, dev)
    clk.stop()
    if train is not None:
        train["clocks"] = clk.summary("train")

    if rank == 0:
        burst, sustained, hbm, src = measured_peaks()
        att_ms = per["attn_fwd"] + per["attn_bwd"]
        ach = FLOP_PER_PAIR * pairs(b_, h_, t_) / (att_ms * 1e-3) / 1e12
        prep_bytes = 302 * b_ * t_ * h_
        line = {
            "metric": METRIC, "value": round(value, 3), "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_max / args.steps, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "cfg1: fused prep + SISA attention fwd+bwd (sisa_fused step)", "B": b_, "T": t_,
                       "H": h_, "d_head": 64, "d_state": 32, "parallelism": f"replicas x{world} (per-rank batch)",
                       "l2": "inputs larger than L2 (proj %.0f MB)" % proj_mb,
                       "flop_per_pair": FLOP_PER_PAIR},
            "roofline": {"kernel": "sisa_attn_fwd + sisa_attn_bwd (tcgen05)", "bound": "tensor",
                         "achieved": round(ach, 3), "peak": burst, "unit": "TFLOP/s", "frac": round(ach / burst, 4),
                         "peak_source": f"{src} bf16 burst",
                         "traffic": round(ATTN_TRAFFIC_PER_UNIT * b_ * h_ * t_),
                         "traffic_note": "ncu DRAM bytes of the three attention kernels per step, scaled from B=1 H=8",
                         "per_call_ms": {k: round(v, 4) for k, v in per.items()},
                         "attn_fwd_tflops": round(FWD_FLOP_PER_PAIR * pairs(b_, h_, t_) / (per["attn_fwd"] * 1e-3) / 1e12, 3),
                         "attn_bwd_tflops": round((FLOP_PER_PAIR - FWD_FLOP_PER_PAIR) * pairs(b_, h_, t_) /
                                                  (per["attn_bwd"] * 1e-3) / 1e12, 3),
                         "prep_fwd_gbs": round(prep_bytes / (per["prep_fwd"] * 1e-3) / 1e9, 1),
                         "hbm_peak_gbs": hbm},
            "e2e": e2e,
            "train": train,
            **extra,
            "gpu_launches": 8 * args.steps,
            "clocks": clk.summary("timed"),
        }
        if not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(H)
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


TRAIN_FLOP_PER_TOKEN = 6 * 151_878_576 + 1152 * 12 * 1024.5 * 12   # matmul params incl. LM head + attention


def run_train(args, rank, world, dev):
    """cfg3: data-parallel training step of the 12-layer model; returns the ``train`` object (rank 0)."""
    import sisa_b200 as sisa
    from sisa_b200 import dp

    cfg = sisa.SISAConfig.preset("sisa-152m", attn_impl="cuda")
    model = dp.build_model(cfg, dev, seed=0)
    trainer = dp.Trainer(model, cuda_graph=not args.train_eager)
    g = torch.Generator(device=dev).manual_seed(100 + rank)
    bt, tt = args.train_batch, 2048
    batches = [torch.randint(0, cfg.vocab_size, (bt, tt), device=dev, generator=g) for _ in range(4)]
    k_steps = max(3, min(args.train_steps, args.steps))
    for i in range(max(args.warmup, 3)):
        trainer.step(batches[i % 4])
    torch.cuda.synchronize(dev)
    if world > 1:
        torch.distributed.barrier()
    s_, e_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s_.record()
    for i in range(k_steps):
        loss = trainer.step(batches[i % 4])
    e_.record()
    torch.cuda.synchronize(dev)
    ms = torch.tensor([s_.elapsed_time(e_)], device=dev)
    if world > 1:
        torch.distributed.all_reduce(ms, op=torch.distributed.ReduceOp.MAX)
    ms = float(ms.item()) / k_steps
    tok_s = world * bt * tt / (ms * 1e-3)
    burst, sustained, _, _ = measured_peaks()
    trainer_buckets = trainer._buckets.bounds if trainer._buckets is not None else []
    trainer.close()                     # the graph holds NCCL work: release it before the group goes
    del trainer, model
    torch.cuda.empty_cache()
    return {"metric": "12L train tokens/s", "value": round(tok_s, 1), "unit": "tokens/s", "n_gpus": world,
            "ms_per_step": round(ms, 3), "steps": k_steps, "per_rank_batch": [bt, tt], "model": "sisa-152m",
            "params": cfg.num_parameters(), "loss_last": round(float(loss), 4),
            "mfu_vs_sustained": round(tok_s * TRAIN_FLOP_PER_TOKEN / (world * sustained * 1e12), 4),
            "parallelism": (f"dp{world} (whole step as one CUDA graph per rank: flat fp32 gradients in "
                            f"{len(trainer_buckets)} buckets, each allreduced by NCCL on a side stream as the "
                            "backward finishes it)" if world > 1 else
                            ("dp1 (eager steps)" if args.train_eager else "dp1 (whole step as one CUDA graph)"))}


def run_e2e(step, dev, args, world):
    """The step end to end through the C ABI with host buffers: every step copies its inputs (proj, z,
    dy) in from pinned host memory and its results (y, d_proj, dz, dlam) back out, inside the timed
    region. Copies and compute are pipelined over two device buffer sets and three streams, as a
    training or serving loop would run them: step k's compute overlaps step k+1's input copy and step
    k-1's output copy (PCIe is full duplex). Events order every reuse of a buffer set."""
    steps = [step, Step(dev, b=step.b, t=step.t, h=step.h, seed=4321)]
    hp = step.proj.cpu().pin_memory()
    hz = step.z.cpu().pin_memory()
    hdy = step.dy.cpu().pin_memory()
    out_dproj = torch.empty(step.dproj.shape, dtype=step.dproj.dtype, pin_memory=True)
    b_, t_, h_ = step.b, step.t, step.h
    out_y = torch.empty((b_, t_, h_ * 64), dtype=torch.bfloat16, pin_memory=True)
    out_dz = torch.empty(step.dz.shape, dtype=torch.float32, pin_memory=True)
    out_dlam = torch.empty((h_,), dtype=torch.float32, pin_memory=True)
    comp = torch.cuda.current_stream(dev)
    cin, cout = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    y_views = [x.o.transpose(1, 2).reshape(b_, t_, h_ * 64) for x in steps]   # views of o's (B, T, H, 64) storage
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_comp = [torch.cuda.Event() for _ in range(2)]
    ev_out = [torch.cuda.Event() for _ in range(2)]
    issued = [0]

    def one():
        k = issued[0]
        i = k % 2
        S = steps[i]
        if k >= 2:
            cin.wait_event(ev_comp[i])      # step k-2 has finished reading this set's inputs
        with torch.cuda.stream(cin):
            S.proj.copy_(hp, non_blocking=True)
            S.z.copy_(hz, non_blocking=True)
            S.dy.copy_(hdy, non_blocking=True)
            ev_in[i].record(cin)
        comp.wait_event(ev_in[i])
        if k >= 2:
            comp.wait_event(ev_out[i])      # step k-2's results have left this set's outputs
        S.run(comp.cuda_stream)
        ev_comp[i].record(comp)
        cout.wait_event(ev_comp[i])
        with torch.cuda.stream(cout):
            out_y.copy_(y_views[i], non_blocking=True)
            out_dproj.copy_(S.dproj, non_blocking=True)
            out_dz.copy_(S.dz, non_blocking=True)
            out_dlam.copy_(S.dlam, non_blocking=True)
            ev_out[i].record(cout)
        issued[0] += 1

    n = max(5, min(args.steps, 20))
    for _ in range(4):
        one()
    torch.cuda.synchronize(dev)
    if world > 1:
        torch.distributed.barrier()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record(cin)
    for _ in range(n):
        one()
    e.record(cout)
    torch.cuda.synchronize(dev)
    ms = torch.tensor([s.elapsed_time(e)], device=dev)
    if world > 1:
        torch.distributed.all_reduce(ms, op=torch.distributed.ReduceOp.MAX)
    ms = float(ms.item())
    h2d = hp.numel() * 2 + hz.numel() * 4 + hdy.numel() * 2
    d2h = out_y.numel() * 2 + out_dproj.numel() * 2 + out_dz.numel() * 4 + out_dlam.numel() * 4
    v = FLOP_PER_PAIR * pairs(b_, h_, t_) * n * world / (ms * 1e-3) / 1e12
    return {"value": round(v, 3), "unit": "TFLOP/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
            "ms_per_step": round(ms / n, 3), "steps": n,
            "pipelining": "2 buffer sets; input copy, compute and output copy on separate streams"}


def cpu_step(heads, seed=0):
    """One fwd+bwd of the reference's pure-PyTorch algorithm (oracle port, fp32) on B=1, `heads` heads, T=4096."""
    from oracle import sisa_oracle as O

    proj, z, lam = O.make_proj_inputs(1, T, heads, seed=seed)
    P = proj.requires_grad_(True)
    Z = z.requires_grad_(True)
    LAM = lam.clone().requires_grad_(True)
    y, _, _ = O.fused_layer(P, Z, LAM, heads, dtype=torch.float32)
    y.backward(torch.ones_like(y))
    return FLOP_PER_PAIR * pairs(1, heads, T)


def cpu_baseline(heads, budget_s=10.0, max_steps=64):
    """The oracle port on the host cores: B=1 x `heads` units at the full T per sample, new seeds, until
    about `budget_s` seconds of CPU work have run (at least two samples)."""
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    cpu_step(heads, seed=1)
    t0 = time.perf_counter()
    n = 0
    flop = 0
    while n < 2 or (time.perf_counter() - t0 < budget_s and n < max_steps):
        flop += cpu_step(heads, seed=2 + n)
        n += 1
    dt = time.perf_counter() - t0
    return {"value": round(flop / dt / 1e12, 5), "unit": "TFLOP/s", "cores": threads, "kind": "port",
            "sample": f"{n} samples of B=1 x H={heads} heads at T=4096 ({B * H // heads} samples make a cfg1 step), "
                      f"fp32, {dt:.1f} s"}


def _ref_import():
    """The reference package (tlstngud/sisa, Triton kernels) from baseline/_ref, or an import error."""
    ref = ROOT / "baseline" / "_ref"
    if not (ref / "sisa").is_dir():
        raise ImportError("baseline/_ref is not installed")
    if str(ref) not in sys.path:
        sys.path.insert(0, str(ref))
    import sisa as sisa_ref   # noqa: F401

    return sisa_ref


def _time_cuda(fn, steps, warmup):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    s_, e_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s_.record()
    for _ in range(steps):
        fn()
    e_.record()
    torch.cuda.synchronize()
    return s_.elapsed_time(e_) / steps


def incumbent_leg(inputs, args):
    """The reference's own GPU path on the same cfg1 inputs: its Triton ``sisa_fused`` forward + backward
    (src/sisa/kernels/fused_prep.py:637) through its autograd function, CUDA-event timed on this GPU."""
    try:
        sisa_ref = _ref_import()
        from sisa.kernels.fused_prep import sisa_fused as ref_fused
    except Exception as e:  # noqa: BLE001
        return {"unavailable": f"reference package: {type(e).__name__}: {e}"[:200]}
    proj, z, lam, dy = inputs
    H = lam.shape[0]
    P = proj.detach().clone().requires_grad_(True)
    Z = z.detach().clone().requires_grad_(True)
    LAM = lam.detach().clone().requires_grad_(True)

    def step():
        y = ref_fused(P, Z, LAM, H)
        y.backward(dy)
        P.grad = Z.grad = LAM.grad = None

    try:
        ms = _time_cuda(step, steps=max(3, min(args.steps, 10)), warmup=2)
    except Exception as e:  # noqa: BLE001
        return {"unavailable": f"reference Triton path failed: {type(e).__name__}: {e}"[:200]}
    b_, t_ = proj.shape[0], proj.shape[1]
    return {"impl": f"reference sisa_fused (Triton, sisa {getattr(sisa_ref, '__version__', '?')}) from baseline/_ref",
            "value": round(FLOP_PER_PAIR * pairs(b_, H, t_) / (ms * 1e-3) / 1e12, 3), "unit": "TFLOP/s",
            "ms_per_step": round(ms, 4), "note": "same inputs as the timed cfg1 step, autograd forward + backward"}


def lce_leg(args, dev, steps=None):
    """cfg2: chunked linear-CE fwd+bwd, hidden [16384 x 1024] bf16 ~ N(0,1), weight [50277 x 1024] fp32
    ~ N(0, 0.02^2) under bf16 autocast, labels uniform. tokens/s and TFLOP/s on 6 N V D, peak memory,
    and the reference's Triton linear-CE on the same inputs."""
    from sisa_b200.kernels.linear_ce import linear_cross_entropy

    N, D, V = args.lce_tokens, 1024, 50277
    g = torch.Generator(device=dev).manual_seed(0)
    h = torch.randn((N, D), generator=g, device=dev).to(torch.bfloat16).requires_grad_(True)
    w = (torch.randn((V, D), generator=g, device=dev) * 0.02).requires_grad_(True)
    lab = torch.randint(0, V, (N,), generator=g, device=dev)

    def make_step(fn):
        def step():
            with torch.autocast("cuda", dtype=torch.bfloat16):
                loss = fn(h, w, lab)
            loss.backward()
            h.grad = None
            w.grad = None
        return step

    k = steps or max(3, min(args.steps, 30))
    step = make_step(linear_cross_entropy)
    for _ in range(max(args.warmup, 2)):
        step()
    torch.cuda.synchronize()
    base = torch.cuda.memory_allocated()
    torch.cuda.reset_peak_memory_stats()
    ms = _time_cuda(step, steps=k, warmup=0)
    peak = torch.cuda.max_memory_allocated() - base
    out = {"metric": "linear-CE fwd+bwd tokens/s (cfg2)", "value": round(N / (ms * 1e-3), 1), "unit": "tokens/s",
           "ms_per_step": round(ms, 3), "tflops": round(6 * N * V * D / (ms * 1e9), 1),
           "peak_mem_mb": round(peak / 2**20, 1), "steps": k, "config": {"N": N, "D": D, "V": V}}
    try:
        _ref_import()
        from sisa.kernels.linear_ce import linear_cross_entropy as ref_lce

        ref_step = make_step(ref_lce)
        for _ in range(2):
            ref_step()
        torch.cuda.synchronize()
        base = torch.cuda.memory_allocated()
        torch.cuda.reset_peak_memory_stats()
        rms = _time_cuda(ref_step, steps=k, warmup=0)
        rpeak = torch.cuda.max_memory_allocated() - base
        out["incumbent"] = {"impl": "reference linear_cross_entropy (Triton) from baseline/_ref",
                            "ms_per_step": round(rms, 3), "value": round(N / (rms * 1e-3), 1), "unit": "tokens/s",
                            "peak_mem_mb": round(rpeak / 2**20, 1)}
    except Exception as e:  # noqa: BLE001
        out["incumbent"] = {"unavailable": f"{type(e).__name__}: {e}"[:200]}
    return out


def run_lce(args):
    dev = torch.device("cuda", 0)
    with Clocks(0) as clk:
        out = lce_leg(args, dev)
    out["clocks"] = clk.summary()
    print(json.dumps(out))


def run_norm(args):
    """The block-boundary norms of one cfg3 block (8 x 2048 tokens, d_model 768, 12 heads) through
    ``block_norm``: the attention norm (residual add, bf16 output, fp32 forget projection) and the
    SwiGLU norm (residual add, two bf16 outputs), forward and backward with every gradient. fp32
    residual stream ~ N(0, 4), bf16 residual ~ N(0, 1). Metric: bytes moved per second (algorithmic)."""
    from sisa_b200.kernels.norm import block_norm

    dev = torch.device("cuda", 0)
    rows, d, nproj = args.norm_rows, 768, 12
    g = torch.Generator(device=dev).manual_seed(0)
    x = (torch.randn((rows, d), generator=g, device=dev) * 2).requires_grad_(True)
    res = torch.randn((rows, d), generator=g, device=dev).to(torch.bfloat16).requires_grad_(True)
    w = (torch.rand((d,), generator=g, device=dev) + 0.5).requires_grad_(True)
    pw = (torch.randn((nproj, d), generator=g, device=dev) * 0.05).requires_grad_(True)
    pb = torch.randn((nproj,), generator=g, device=dev).requires_grad_(True)
    bf = torch.bfloat16
    g_attn = [torch.randn((rows, d), generator=g, device=dev), torch.randn((rows, d), generator=g, device=dev).to(bf),
              torch.randn((rows, nproj), generator=g, device=dev)]
    g_ffn = [torch.randn((rows, d), generator=g, device=dev)] + \
        [torch.randn((rows, d), generator=g, device=dev).to(bf) for _ in range(2)]

    def step():
        a = block_norm(x, w, 1e-6, res=res, out_dtypes=(bf,), proj=(pw, pb))
        torch.autograd.backward(list(a), g_attn)
        f = block_norm(x, w, 1e-6, res=res, out_dtypes=(bf, bf))
        torch.autograd.backward(list(f), g_ffn)
        for t in (x, res, w, pw, pb):
            t.grad = None

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()      # replayed, so that the time is the kernels' and not the host's
    with torch.cuda.graph(graph):
        step()
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    k = max(3, min(args.steps, 50))
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(k)]
    with Clocks(0) as clk:
        for i in range(k):
            flush.zero_()   # inputs are 75 MB per norm: flush L2 between steps
            ev[i][0].record()
            graph.replay()
            ev[i][1].record()
        torch.cuda.synchronize()
    ms = sum(a.elapsed_time(b) for a, b in ev) / k
    # algorithmic bytes per row: attention norm fwd 9268 + bwd 12340, SwiGLU norm fwd 10756 + bwd 13828
    per_row = (3072 + 1536 + 3072 + 1536 + 48 + 4) + (3072 + 1536 + 3072 + 48 + 4 + 3072 + 1536) + \
        (3072 + 1536 + 3072 + 2 * 1536 + 4) + (3072 + 2 * 1536 + 3072 + 4 + 3072 + 1536)
    print(json.dumps({"metric": "block-boundary RMSNorm fwd+bwd (attention and SwiGLU norms of one cfg3 block)",
                      "value": round(rows * per_row / (ms * 1e-3) / 1e9, 1), "unit": "GB/s",
                      "ms_per_step": round(ms, 4), "steps": k, "dtype": "fp32 stream, bf16 outputs",
                      "config": {"rows": rows, "d": d, "n_proj": nproj, "bytes_per_row": per_row,
                                 "l2": "flushed between steps", "timing": "CUDA graph replay of the step"},
                      "clocks": clk.summary()}))


def decode_leg(args, dev, steps=None):
    """cfg4: 12-layer sisa-152m, random init, bf16 weights; batch 64, prompt 8192 ids (id 0 first), then
    greedy decode steps. Prefill tokens/s and per-step decode latency (CUDA-graph replay of the whole step)
    with the cache and weight bytes read per step."""
    import sisa_b200 as sisa
    from sisa_b200.generation import DecodeGraph, SISACache

    Bd, P = args.decode_batch, args.decode_prompt
    S = steps or args.decode_steps
    if S < 10:
        raise ValueError("decode steps must be >= 10 (1 + 4 eager, 2 warm-up graph steps, then timed steps)")
    cfg = sisa.SISAConfig.preset("sisa-152m", attn_impl="cuda")
    torch.manual_seed(0)
    model = sisa.SISAForCausalLM(cfg).to(dev).to(torch.bfloat16).eval()
    g = torch.Generator(device=dev).manual_seed(1)
    ids = torch.randint(0, cfg.vocab_size, (Bd, P), generator=g, device=dev)
    ids[:, 0] = 0
    with torch.no_grad():
        # warm-up at the full size: the kernels, and the caching allocator's blocks for the prompt's
        # activations and a cache of the same capacity, so the timed prefill allocates from those blocks
        # instead of timing device allocations
        model(ids, cache=SISACache(capacity=P + S + 1), logits_to_keep=1)
        torch.cuda.synchronize()
        cache = SISACache(capacity=P + S + 1)
        s_, e_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s_.record()
        logits = model(ids, cache=cache, logits_to_keep=1).logits[:, -1]
        e_.record()
        torch.cuda.synchronize()
        prefill_ms = s_.elapsed_time(e_)
        nxt = logits.float().argmax(-1)
        # eager steps (every kernel dispatched from Python), the first on the graph's capture stream
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            logits = model(nxt.unsqueeze(1), cache=cache, logits_to_keep=1).logits[:, -1]
            nxt = logits.float().argmax(-1)
        torch.cuda.current_stream(dev).wait_stream(side)
        n_eager = 4
        s_.record()
        for _ in range(n_eager):
            logits = model(nxt.unsqueeze(1), cache=cache, logits_to_keep=1).logits[:, -1]
            nxt = logits.float().argmax(-1)
        e_.record()
        torch.cuda.synchronize()
        eager_ms = s_.elapsed_time(e_) / n_eager
        # the same step captured once as a CUDA graph (generate's default) and replayed per token
        graph = DecodeGraph(model, cache, Bd, stream=side)
        for _ in range(2):
            nxt = graph.step(nxt).float().argmax(-1)
        torch.cuda.synchronize()
        n = S - 3 - n_eager
        s_.record()
        for _ in range(n):
            nxt = graph.step(nxt).float().argmax(-1)
        e_.record()
        torch.cuda.synchronize()
        step_ms = s_.elapsed_time(e_) / n
        graph.close()
    del cache, model
    L_avg = P + 3 + n_eager + n / 2
    per_tok = cfg.n_layer * cfg.n_head * (64 * 2 * 2 + 32 * 2 + 8)   # k, v, b~ (bf16) + g, F (fp32)
    cache_bytes = Bd * L_avg * per_tok
    weight_bytes = 2 * (cfg.num_parameters())
    return {"metric": "decode step latency (cfg4)", "value": round(step_ms, 3), "unit": "ms/step",
            "prefill_tokens_s": round(Bd * P / (prefill_ms * 1e-3), 1), "prefill_ms": round(prefill_ms, 1),
            "decode_steps_timed": n, "eager_ms_per_step": round(eager_ms, 3),
            "timing": "CUDA graph replay of the whole decode step (DecodeGraph)",
            "cache_bytes_per_step": int(cache_bytes),
            "hbm_gbs": round((cache_bytes + weight_bytes) / (step_ms * 1e-3) / 1e9, 1),
            "config": {"batch": Bd, "prompt": P, "new_tokens": S, "model": "sisa-152m"}}


def gemm_leg(args, dev, n=8192, steps=None):
    """The CTA-pair tcgen05 GEMM (``sisa_gemm``) on C = A B^T, A and B (n x n) bf16 K-major, bf16 C,
    in each tile shape and as the cost model chooses, next to cuBLAS (``torch.mm``) on the same
    operands (384 MB at n = 8192, more than L2). TFLOP/s on 2 n^3."""
    from sisa_b200.kernels.gemm import matmul_t

    g = torch.Generator(device=dev).manual_seed(0)
    a = torch.randn((n, n), generator=g, device=dev).to(torch.bfloat16)
    b = torch.randn((n, n), generator=g, device=dev).to(torch.bfloat16)
    c = torch.empty((n, n), device=dev, dtype=torch.bfloat16)
    k = steps or max(3, min(args.steps, 50))
    out = {"metric": "GEMM TFLOP/s (C = A B^T, bf16)", "unit": "TFLOP/s", "config": {"n": n}, "steps": k}
    prev = os.environ.get("SISA_GEMM_TILE")
    try:
        for name, tile in (("narrow", "narrow"), ("wide", "wide"), ("auto", None)):
            if tile:
                os.environ["SISA_GEMM_TILE"] = tile
            else:
                os.environ.pop("SISA_GEMM_TILE", None)
            ms = _time_cuda(lambda: matmul_t(a, b, c), steps=k, warmup=max(args.warmup, 2))
            out[name] = round(2 * n ** 3 / (ms * 1e9), 1)
    finally:
        if prev is None:
            os.environ.pop("SISA_GEMM_TILE", None)
        else:
            os.environ["SISA_GEMM_TILE"] = prev
    ms = _time_cuda(lambda: torch.mm(a, b.t(), out=c), steps=k, warmup=max(args.warmup, 2))
    out["cublas"] = round(2 * n ** 3 / (ms * 1e9), 1)
    out["value"] = out["auto"]
    return out


def run_gemm(args):
    dev = torch.device("cuda", 0)
    with Clocks(0) as clk:
        out = gemm_leg(args, dev, n=args.gemm_size)
    out["clocks"] = clk.summary()
    print(json.dumps(out))


def run_train_only(args):
    """Only the config 3 training leg (the whole step as one CUDA graph per rank); under torchrun one
    rank per GPU, data-parallel, like the train leg of the default run."""
    rank, world, local = dist_setup(args.gpus)
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    with Clocks(local) as clk:
        with clk.window("train"):
            out = run_train(args, rank, world, dev)
    out["clocks"] = clk.summary("train")
    if rank == 0:
        print(json.dumps(out))
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


def run_decode(args):
    dev = torch.device("cuda", 0)
    with Clocks(0) as clk:
        out = decode_leg(args, dev)
    out["clocks"] = clk.summary()
    print(json.dumps(out))


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    heads = args.cpu_sample_heads
    for _ in range(args.warmup):
        cpu_step(heads, seed=0)
    t0 = time.perf_counter()
    flop = 0
    for k in range(args.steps):
        flop += cpu_step(heads, seed=1 + k)
    dt = time.perf_counter() - t0
    value = flop / dt / 1e12
    line = {"metric": METRIC, "value": round(value, 5), "unit": "TFLOP/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(dt / args.steps * 1e3, 2), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic", "impl": "reference",
            "config": {"workload": "cfg1: fused prep + SISA attention fwd+bwd (sisa_fused step)", "B": B, "T": T,
                       "H": H, "d_head": 64, "d_state": 32},
            "cpu_baseline": {"value": round(value, 5), "unit": "TFLOP/s", "cores": threads, "kind": "port",
                             "sample": f"each step B=1 x H={heads} at T=4096, fp32 pure-PyTorch CPU algorithm"},
            "e2e": {"value": round(value, 5), "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["cuda", "reference"], default="cuda")
    ap.add_argument("--cpu-sample-heads", type=int, default=4)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-train", action="store_true")
    ap.add_argument("--no-extra", action="store_true",
                    help="skip the config 2 / config 4 legs and the reference Triton incumbent of the default run")
    ap.add_argument("--extra-decode-steps", type=int, default=48, help="decode steps of the default run's cfg4 leg")
    ap.add_argument("--workload", choices=["attn", "lce", "decode", "norm", "gemm", "train"], default="attn",
                    help="attn (default: config 1 + the config 3 training leg), lce (config 2), decode (config 4), "
                         "norm (the fused block-boundary norms of config 3), gemm (the CTA-pair GEMM against "
                         "cuBLAS), train (the config 3 training leg alone)")
    ap.add_argument("--gemm-size", type=int, default=8192)
    ap.add_argument("--norm-rows", type=int, default=16384)
    ap.add_argument("--lce-tokens", type=int, default=16384, help="hidden rows of the lce workload (cfg2: 16384)")
    ap.add_argument("--decode-batch", type=int, default=64)
    ap.add_argument("--decode-prompt", type=int, default=8192)
    ap.add_argument("--decode-steps", type=int, default=256)
    ap.add_argument("--train-steps", type=int, default=20)
    ap.add_argument("--train-batch", type=int, default=8)
    ap.add_argument("--train-eager", action="store_true",
                    help="train leg without the CUDA graph (for kernel launch lists: ncu cannot follow the capture)")
    ap.add_argument("--B", type=int, default=B, help="batch (default: config 1)")
    ap.add_argument("--T", type=int, default=T, help="sequence length (default: config 1)")
    ap.add_argument("--H", type=int, default=H, help="heads (default: config 1)")
    args = ap.parse_args(argv)
    if args.impl == "reference":
        run_reference(args)
    elif args.workload == "lce":
        run_lce(args)
    elif args.workload == "decode":
        run_decode(args)
    elif args.workload == "norm":
        run_norm(args)
    elif args.workload == "gemm":
        run_gemm(args)
    elif args.workload == "train":
        run_train_only(args)
    else:
        run_cuda(args)


if __name__ == "__main__":
    main()
