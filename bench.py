"""Sampler benchmark: sampled rows/s and logits GB/s (fraction of HBM peak).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload: 4096 rows x 151,936 f32 logits (Qwen2.5-0.5B vocab), distribution of
workload 5 (N(0, 2.5^2) + row offset + 8 peaks), temp 0.7, top-k 50, top-p 0.9,
one xorshift64* draw per row.  Synthetic data: no model or dataset exists here.

One step = one zs_sample call over the rank's 4096 rows: the streaming select
kernel (zs_wselect_kernel: every row of this workload has a top-50 shortlist)
and the per-row merge kernel.  Each step is also timed on its own (per_step_ms).
With N GPUs (torchrun, one process per GPU) every rank samples its own 4096
rows (row split, no communication): weak scaling, value = N*4096 rows / max
over ranks of the step time.  For N > 1 the vocab-sharded mode over the same
4096 rows (partials -> row-owner exchange or all-gather -> merge) is reported
beside it, with its partials / merge / exchange split.

With one GPU the line also carries: by_config (the five workloads at their own
batch sizes 1, 256, 1024, 512 and 4096, each with the select / merge split and
the parity counts of one checked call against the restatement and the unchanged
reference), host_api_b1 (zen::sample_token on one host row, the drop-in C++
API), the logits display numbers, the decode loop, the lm_head routes and the
full-vocabulary nucleus.

Inputs (2.49 GB per rank) are larger than L2 (126 MB), so every step reads HBM;
smaller workloads rotate over copies of their input that together exceed L2.
"""

from __future__ import annotations

import argparse
import json
import os
import re
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

V = 151936
ROWS = 4096
WORKLOAD = 5
ROW_BYTES = V * 4
METRIC = "sampled rows/sec & logits GB/s (% of HBM peak) at batch 1/256/4096, 1-8 B200"
UNIT = "rows/s"
FALLBACK_HBM_GBS = 6650.0


def env_int(name, default):
    try:
        return int(os.environ.get(name, default))
    except ValueError:
        return default


def hbm_peak():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def committed_traffic(rows):
    """dram bytes per launch of the select kernel on this workload, from the
    committed ncu summary (profiles/), scaled to `rows` rows; None if absent."""
    path = os.path.join(ROOT, "profiles", "zs_wselect_kernel_workload5.md")
    try:
        txt = open(path).read()
    except OSError:
        return None
    m = re.search(r"traffic_bytes_per_row:\s*([0-9.eE+]+)", txt)
    return float(m.group(1)) * rows if m else None


class ClockSampler:
    """SM clocks and clock-event (throttle) reasons sampled during the timed region:
    NVML read every 2 ms from a thread (the timed region of a short run lasts only
    milliseconds), else nvidia-smi every 100 ms.  Reads only; changes nothing."""
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    # nvmlClocksEventReason* bits
    REASONS = {0x8: "hw_slowdown", 0x40: "hw_thermal_slowdown", 0x20: "sw_thermal_slowdown",
               0x4: "sw_power_cap"}

    def __init__(self, gpu_index, pci_bus_id=None):
        self.gpu = gpu_index
        self.pci = pci_bus_id
        self.proc = None
        self.path = None
        self.thread = None
        self.stop_flag = False
        self.sm, self.mx, self.reasons = [], [], set()
        self.err = None

    def _nvml_sample(self, nv, h, mx):
        self.sm.append(float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)))
        self.mx.append(float(mx))
        try:
            bits = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
        except Exception as e:  # clocks are still recorded; say why reasons are not
            self.err = f"clock event reasons: {e}"
            return
        for bit, name in self.REASONS.items():
            if bits & bit:
                self.reasons.add(name)

    def _nvml_loop(self, nv, h, mx):
        while not self.stop_flag:
            try:
                self._nvml_sample(nv, h, mx)
            except Exception as e:
                self.err = f"nvml: {e}"
                break
            time.sleep(0.002)

    def start(self):
        try:
            import threading
            import pynvml as nv
            nv.nvmlInit()
            h = None
            if self.pci:
                try:
                    h = nv.nvmlDeviceGetHandleByPciBusId(self.pci)
                except Exception:
                    h = None
            if h is None:
                h = nv.nvmlDeviceGetHandleByIndex(self.gpu)
            mx = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
            self._nvml_sample(nv, h, mx)  # one sample before the timed region starts
            self.nv, self.h, self.mx_clock = nv, h, mx
            self.thread = threading.Thread(target=self._nvml_loop, args=(nv, h, mx), daemon=True)
            self.thread.start()
            return
        except Exception as e:
            self.err = f"nvml unavailable: {e}"
            self.thread = None
            self.sm, self.mx, self.reasons = [], [], set()
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.QUERY}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        out = {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        if self.thread is not None:
            try:  # one sample as the timed region ends, whatever the thread managed
                self._nvml_sample(self.nv, self.h, self.mx_clock)
            except Exception as e:
                self.err = f"nvml: {e}"
            self.stop_flag = True
            self.thread.join(timeout=5)
            src = "nvml, every 2 ms"
        elif self.proc is not None:
            # nvidia-smi needs a moment to start: wait (up to 3 s) for its first line
            t_end = time.monotonic() + 3.0
            while time.monotonic() < t_end:
                try:
                    if os.path.getsize(self.path) > 0:
                        break
                except OSError:
                    break
                time.sleep(0.05)
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
            try:
                for line in open(self.path):
                    parts = [p.strip() for p in line.split(",")]
                    if len(parts) < 9:
                        continue
                    try:
                        self.sm.append(float(parts[1]))
                        self.mx.append(float(parts[2]))
                    except ValueError:
                        continue
                    for n, v in zip(names, parts[5:9]):
                        if v.lower() == "active":
                            self.reasons.add(n)
                os.unlink(self.path)
            except OSError:
                pass
            src = "nvidia-smi, every 100 ms"
        else:
            if self.err:
                out["note"] = self.err
            return out
        if self.sm:
            out = {"sm_mhz": statistics.median(self.sm), "sm_max_mhz": max(self.mx),
                   "sm_min_mhz": min(self.sm), "reasons": sorted(self.reasons),
                   "samples": len(self.sm), "source": src}
        if self.err:
            out["note"] = self.err
        return out


def cpu_reference_rate(x_rows, params, seeds, budget_s=10.0, nthreads=None):
    """The reference's own sampler (oracle/_ref, src/sample.cpp compiled unchanged)
    on the host cores: rows/s over a bounded sample of the workload rows (whole
    passes over the batch, or a prefix of it, for about budget_s seconds)."""
    import oracle
    nthreads = nthreads or (os.cpu_count() or 1)
    probe = min(len(x_rows), max(64, nthreads * 4))
    t0 = time.perf_counter()
    oracle.reference_sample(x_rows[:probe], params, seeds[:probe], nthreads=nthreads)
    rate = probe / max(time.perf_counter() - t0, 1e-9)
    chunk = int(min(len(x_rows), max(probe, rate * budget_s)))
    done, t0 = 0, time.perf_counter()
    while True:
        oracle.reference_sample(x_rows[:chunk], params, seeds[:chunk], nthreads=nthreads)
        done += chunk
        dt = time.perf_counter() - t0
        if dt >= budget_s or chunk < len(x_rows):
            break
    return done / dt, done, dt, nthreads


def lmhead_bench(s, dev, stream, hbm_peak):
    import numpy as np
    import torch
    from zeninfer_b200 import SamplingParams, states_to_tensor
    E = 896
    g = torch.Generator(device=dev).manual_seed(17)
    W = (torch.randn(V, E, device=dev, generator=g) * 0.05).to(torch.bfloat16)
    nw = torch.rand(E, device=dev, generator=g) + 0.5
    p = SamplingParams(temp=0.7, top_k=50, top_p=0.9)
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            tf_peak, tf_kind = float(json.load(f)["bf16_tflops"]), "measured burst"
    except Exception:
        tf_peak, tf_kind = 1590.0, "fallback"
    out = {"weights": "bf16 [151936][896], seeded N(0, 0.05^2)", "hidden": "N(0, 3^2) f32",
           "params": "temp 0.7, top-k 50, top-p 0.9"}
    for B in (4096, 2048, 1024, 512, 256, 8, 1):
        h = torch.randn(B, E, device=dev, generator=g) * 3
        st = states_to_tensor([i + 1 for i in range(B)], dev)
        ids = torch.empty(B, dtype=torch.int32, device=dev)
        fused = lambda: s.lmhead_sample(h, nw, W, p, st, out=ids, stream=stream)
        reps = 10 if B > 1 else 100
        # the default route (exact up to 8 rows, two passes below 1024, fused from 1024) ...
        for _ in range(3):
            fused()
        torch.cuda.synchronize()
        ms_auto = time_device_steps(fused, reps, stream) / reps
        # ... and the fused route forced, with its kernels timed one by one
        s.set_lmhead_route("fused")
        for _ in range(3):
            fused()
        torch.cuda.synchronize()
        s.set_timing(True)
        s.get_timing()
        ms = time_device_steps(fused, reps, stream) / reps
        kt = s.get_timing()
        s.set_timing(False)
        # the other tiling (one-CTA tiles where the default pairs CTAs, and back)
        other = "single" if B >= 512 else "pair"
        s.set_lmhead_tiles(other)
        for _ in range(3):
            fused()
        torch.cuda.synchronize()
        s.set_timing(True)
        s.get_timing()
        ms_other = time_device_steps(fused, reps, stream) / reps
        kt_other = s.get_timing()
        s.set_timing(False)
        s.set_lmhead_tiles("auto")
        s.set_lmhead_route("auto")
        k_ms = kt["lmhead_ms"] / max(1, kt["lmhead_launches"])
        xn = torch.nn.functional.rms_norm(h, (E,), nw, 1e-6).to(torch.bfloat16)

        def unfused():
            lg = torch.mm(xn, W.t(), out_dtype=torch.float32)
            s.sample(lg, p, st, out=ids, stream=stream)
        for _ in range(3):
            unfused()
        torch.cuda.synchronize()
        ms_u = time_device_steps(unfused, reps, stream) / reps
        lg_own = torch.empty((B, V), dtype=torch.float32, device=dev)

        def two_pass():  # this library's tcgen05 GEMM writing logits, then zs_sample
            s.lmhead_logits(h, nw, W, out=lg_own, stream=stream)
            s.sample(lg_own, p, st, out=ids, stream=stream)
        s.set_lmhead_route("two_pass")  # tensor-core logits (not the exact route)
        for _ in range(3):
            two_pass()
        torch.cuda.synchronize()
        ms_t = time_device_steps(two_pass, reps, stream) / reps
        s.set_lmhead_route("auto")
        del lg_own
        flops = 2.0 * B * E * V
        wbytes = V * E * 2 + B * E * 2
        r = {"default_route_us_per_call": ms_auto * 1e3,
             "default_route": "exact" if B <= 8 else ("two_pass" if B < 1024 else "fused"),
             "tiles": "cta_pair_256x256" if B >= 512 else "cta_128x128",
             "us_per_call": ms * 1e3, "rows_per_s": B / (ms / 1e3),
             "kernel_us": k_ms * 1e3,
             "other_tiles": {"tiles": other, "us_per_call": ms_other * 1e3,
                             "kernel_us": kt_other["lmhead_ms"]
                             / max(1, kt_other["lmhead_launches"]) * 1e3},
             "rmsnorm_us": kt["lmnorm_ms"] / max(1, kt["lmnorm_launches"]) * 1e3,
             "merge_us": kt["merge_ms"] / max(1, kt["merge_launches"]) * 1e3,
             "unfused_cublas_plus_zs_sample_us": ms_u * 1e3,
             "two_pass_own_gemm_plus_zs_sample_us": ms_t * 1e3}
        if B > 1:
            r["roofline"] = {"bound": "tensor", "achieved": flops / (k_ms / 1e3) / 1e12,
                             "peak": tf_peak, "unit": "TFLOP/s",
                             "frac": flops / (k_ms / 1e3) / 1e12 / tf_peak,
                             "peak_source": f"bf16_tflops, {tf_kind}",
                             "algorithmic_flops_per_launch": flops}
        else:
            r["roofline"] = {"bound": "hbm", "achieved": wbytes / (k_ms / 1e3) / 1e9,
                             "peak": hbm_peak, "unit": "GB/s",
                             "frac": wbytes / (k_ms / 1e3) / 1e9 / hbm_peak,
                             "algorithmic_bytes_per_launch": wbytes}
        out[f"b{B}"] = r
        del h
    try:
        import oracle
        if oracle.have_reference():
            n = 4
            hc = (torch.randn(n, E, generator=torch.Generator().manual_seed(3)) * 3).numpy()
            wf = W.float().cpu().numpy()
            nth = os.cpu_count() or 1
            t0 = time.perf_counter()
            _, lg = oracle.reference_lmhead(hc, nw.cpu().numpy(), 1e-6, wf, impl=1, nthreads=nth)
            oracle.reference_sample(lg, p, np.arange(1, n + 1, dtype=np.uint64), nthreads=nth)
            dt = time.perf_counter() - t0
            out["cpu_reference"] = {"rows_per_s": n / dt, "cores": nth, "kind": "reference",
                                    "sample": f"{n} rows: zen::rmsnorm + zen::matvec_f32 (AVX2) "
                                              "+ zen::sample_token, src/ compiled unchanged"}
            # Ids of the fused route (bf16 xn and weights, f32 accumulation) against the
            # reference's own f32 lm_head + sample_token on the same rows and seeds.
            n = 64
            hc = (torch.randn(n, E, generator=torch.Generator().manual_seed(4)) * 3)
            cmp = {"rows": n, "precision": "fused route: xn rounded to bf16, bf16 weights, f32 "
                                           "accumulation; reference: f32 xn and f32 matvec over "
                                           "the same (bf16-valued) weights"}
            s.set_lmhead_route("fused")
            try:
                for label, pp in (("sampled", p), ("greedy", SamplingParams())):
                    st_n = states_to_tensor([i + 1 for i in range(n)], dev)
                    got = s.lmhead_sample(hc.to(dev), nw, W, pp, st_n, stream=stream)
                    torch.cuda.synchronize()
                    got = got.cpu().numpy()
                    _, lg = oracle.reference_lmhead(hc.numpy(), nw.cpu().numpy(), 1e-6, wf,
                                                    impl=1, nthreads=nth)
                    ref, _ = oracle.reference_sample(lg, pp, np.arange(1, n + 1, dtype=np.uint64),
                                                     nthreads=nth)
                    cmp[f"{label}_id_mismatch_vs_reference_f32"] = int((got != ref).sum())
            finally:
                s.set_lmhead_route("auto")
            out["parity_vs_reference_f32"] = cmp
            # The exact route (the default up to 4 rows): logits against the
            # reference's f32 lm_head bit for bit, ids against its sample_token.
            ne = 4
            he = hc[:ne]
            ex = {"rows": ne, "precision": "exact route: f32 xn, f32 fused multiply-adds in "
                                           "the reference's AVX2 summation order"}
            s.set_lmhead_route("exact")
            try:
                lg_dev = s.lmhead_logits(he.to(dev), nw, W, eps=1e-6, stream=stream)
                st_e = states_to_tensor([i + 1 for i in range(ne)], dev)
                got = s.lmhead_sample(he.to(dev), nw, W, p, st_e, stream=stream)
                torch.cuda.synchronize()
                _, lg = oracle.reference_lmhead(he.numpy(), nw.cpu().numpy(), 1e-6, wf, impl=1,
                                                nthreads=nth)
                ref, _ = oracle.reference_sample(lg, p, np.arange(1, ne + 1, dtype=np.uint64),
                                                 nthreads=nth)
                mism = lg_dev.cpu().numpy().view(np.uint32) != lg.view(np.uint32)
                ex["logit_bit_mismatch_vs_reference_f32"] = int(mism.sum())
                ex["sampled_id_mismatch_vs_reference_f32"] = int((got.cpu().numpy() != ref).sum())
            finally:
                s.set_lmhead_route("auto")
            out["exact_route_vs_reference_f32"] = ex
    except Exception as e:  # reported, never fatal
        out["cpu_reference"] = {"note": str(e)}
    del W
    torch.cuda.synchronize()
    return out


def full_vocab_top_p_bench(s, dev, stream):
    import numpy as np
    import torch
    from zeninfer_b200 import SamplingParams, states_to_tensor
    from zeninfer_b200 import workloads as W
    rows = 1024
    wl = W.WORKLOADS[3]
    p = SamplingParams(temp=1.0, top_k=V, top_p=0.95)
    xh = W.generate(3, rows)
    x = torch.from_numpy(xh).to(dev)
    st = states_to_tensor(wl.row_states(0, rows), dev)
    ids = torch.empty(rows, dtype=torch.int32, device=dev)
    fn = lambda: s.sample(x, p, st, out=ids, stream=stream)
    fn()
    torch.cuda.synchronize()
    reps = 3
    ms = time_device_steps(fn, reps, stream) / reps
    res = s.sample(x[:64], p, states_to_tensor(wl.row_states(0, 64), dev), row_info=True,
                   stream=stream)
    m = res.row_info["m"]
    out = {"rows": rows, "params": "temp 1.0, top-p 0.95, top_k = n_vocab (151,936)",
           "ms_per_call": ms, "rows_per_s": rows / (ms / 1e3),
           "nucleus_size_median": float(np.median(m))}
    try:
        import oracle
        if oracle.have_reference():
            n = 32
            nth = os.cpu_count() or 1
            t0 = time.perf_counter()
            oracle.reference_sample(xh[:n], p, wl.row_seeds(0, n), nthreads=nth)
            dt = time.perf_counter() - t0
            out["cpu_reference"] = {"rows_per_s": n / dt, "cores": nth, "kind": "reference",
                                    "sample": f"{n} rows, zen::sample_token with top_k = n"}
    except Exception as e:  # reported, never fatal
        out["cpu_reference"] = {"note": str(e)}
    del x
    return out


def run_reference_arm(args, rank, world):
    """--impl reference: zeninfer's CPU sampler on the host cores, same workload."""
    if rank != 0:
        return
    import numpy as np
    import oracle
    from zeninfer_b200 import workloads as W
    if not oracle.have_reference():
        print(json.dumps({"impl": "reference", "unavailable":
                          "oracle/_ref/libzen_ref.so not built (needs the reference sources)"}))
        return
    wl = W.WORKLOADS[WORKLOAD]
    nthreads = os.cpu_count() or 1
    x = W.generate(WORKLOAD, ROWS)
    seeds = wl.row_seeds(0, ROWS)
    # Calibrate one step to a bounded sample: at most 3 s of host work, and the
    # whole warm-up + timed run within about two minutes.
    t0 = time.perf_counter()
    probe = min(ROWS, max(64, 4 * nthreads))
    oracle.reference_sample(x[:probe], wl.params, seeds[:probe], nthreads=nthreads)
    rate = probe / max(time.perf_counter() - t0, 1e-9)
    step_s = min(3.0, 120.0 / max(1, args.steps + args.warmup))
    step_rows = int(min(ROWS, max(nthreads, rate * step_s)))
    for _ in range(args.warmup):
        oracle.reference_sample(x[:step_rows], wl.params, seeds[:step_rows], nthreads=nthreads)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        oracle.reference_sample(x[:step_rows], wl.params, seeds[:step_rows], nthreads=nthreads)
        times.append(time.perf_counter() - t0)
    total = sum(times)
    value = step_rows * len(times) / total
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * total / len(times),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32/f64",
        "data": "synthetic",
        "config": {"workload": "4096 x 151936 f32 logits, temp 0.7, top-k 50, top-p 0.9",
                   "rows_per_step": step_rows},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": nthreads, "kind": "reference",
                         "sample": f"{step_rows} of the 4096 rows per step, zen::sample_token "
                                   f"per row on {nthreads} host threads"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def time_device_steps(fn, steps, stream, per_step=None):
    """Device time (ms) of `steps` calls of fn on `stream`, by CUDA events around the
    whole run; with a list as per_step, each step's own time (ms) is appended to it
    (an event after every step)."""
    import torch
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    marks = []
    start.record(stream)
    for _ in range(steps):
        fn()
        if per_step is not None:
            ev = torch.cuda.Event(enable_timing=True)
            ev.record(stream)
            marks.append(ev)
    end.record(stream)
    end.synchronize()
    if per_step is not None:
        prev = start
        for ev in marks:
            per_step.append(prev.elapsed_time(ev))
            prev = ev
    return start.elapsed_time(end)


def spread(ms_list):
    """min / median / max of per-step times (ms)."""
    if not ms_list:
        return None
    return {"min_ms": min(ms_list), "median_ms": statistics.median(ms_list),
            "max_ms": max(ms_list), "n": len(ms_list)}


L2_BYTES = 126 * 2**20


def shortlist_len(p):
    if p.temp <= 0:
        return 0
    return min(p.top_k, V) if p.top_k > 0 else min(256, V)


def parity_counts(s, dev, x, p, states, seeds, stream):
    """One checked call outside the timed region, against the restatement (oracle/)
    and the unchanged reference (oracle/_ref, src/sample.cpp): the counts the parity
    rules name.  Returns a dict; never raises."""
    import numpy as np
    import torch
    from zeninfer_b200 import Rng, states_to_tensor, tensor_to_states
    try:
        import oracle
        k = shortlist_len(p)
        xd = torch.from_numpy(x).to(dev)
        st = states_to_tensor(states, dev)
        res = s.sample(xd, p, st, row_info=True, cand_ld=k, stream=stream)
        torch.cuda.synchronize()
        g_ids = res.ids.cpu().numpy()
        g_st = tensor_to_states(st)
        # the timed call wants ids only, which takes the certified parallel tail:
        # it must give the same ids and states as this checked call
        st2 = states_to_tensor(states, dev)
        t_ids = s.sample(xd, p, st2, stream=stream).ids
        torch.cuda.synchronize()
        t_ids = t_ids.cpu().numpy()
        t_st = tensor_to_states(st2)
        o_st = np.array(states, dtype=np.uint64, copy=True)
        o_ids, o_info, o_cid, _, o_cp = oracle.oracle_sample(x, p, o_st, cand_ld=k)
        greedy = p.temp <= 0
        near = (o_info["boundary"] < 1e-6) if not greedy else np.zeros(len(g_ids), bool)
        out = {"rows": int(len(g_ids)),
               "boundary_rows": int(near.sum()),
               "boundary_rows_id_differs": int(((g_ids != o_ids) & near).sum()),
               "id_mismatch_vs_restatement": int(((g_ids != o_ids) & ~near).sum()),
               "rng_state_mismatch_vs_restatement": int((g_st != o_st).sum()),
               "timed_call_id_mismatch": int((t_ids != g_ids).sum()),
               "timed_call_rng_mismatch": int((t_st != g_st).sum())}
        if k > 0:
            gc = res.cand_ids.cpu().numpy()
            gp = res.cand_probs.cpu().numpy()
            kk = np.minimum(o_info["k"], k)
            sets = 0
            rel = 0.0
            for r in range(len(g_ids)):
                n = int(kk[r])
                if not np.array_equal(gc[r, :n], o_cid[r, :n]):
                    sets += 1
                op = o_cp[r, :n]
                m = op > 0
                if m.any():
                    rel = max(rel, float(np.max(np.abs(gp[r, :n][m] - op[m]) / op[m])))
            out["topk_mismatch_vs_restatement"] = sets
            out["max_rel_prob_err"] = rel
        if oracle.have_reference():
            ref_ids, ref_next = oracle.reference_sample(x, p, seeds)
            diff = g_ids != ref_ids
            rows = np.nonzero(diff)[0]
            tie = np.zeros(len(g_ids), bool)
            tie[rows] = x[rows, ref_ids[rows]] == x[rows, g_ids[rows]]
            out["id_mismatch_vs_reference"] = int((diff & ~tie & ~near).sum())
            out["tie_group_rows"] = int((diff & tie).sum())
            nxt = []
            for v in g_st:
                r = Rng(0)
                r.state = int(v)
                nxt.append(r.next())
            out["rng_mismatch_vs_reference"] = int((np.array(nxt, dtype=np.uint64) != ref_next).sum())
            if greedy:
                out["greedy_mismatch_vs_reference"] = int(diff.sum())
        return out
    except Exception as e:  # reported, never fatal
        return {"error": str(e)}


def config_bench(s, dev, stream, peak, row0=0, with_parity=True, only=None):
    """BASELINE's five workloads at their own batch sizes (workloads 1 and 4 also
    greedy): device time per call, the select / merge split, GB/s against the HBM
    peak, and the parity counts of one checked call.  Small inputs rotate over
    copies that together exceed L2 (126 MB), so every call reads HBM."""
    import torch
    from zeninfer_b200 import SamplingParams, states_to_tensor
    from zeninfer_b200 import workloads as W
    out = {}
    for cfg, wl in W.WORKLOADS.items():
        if only is not None and cfg not in only:
            continue
        B = wl.batch
        xh = W.generate(cfg, B, row0=row0)
        copies = max(1, -(-2 * L2_BYTES // (B * ROW_BYTES))) if B * ROW_BYTES < 2 * L2_BYTES else 1
        X = torch.empty((copies, B, V), dtype=torch.float32, device=dev)
        X[0].copy_(torch.from_numpy(xh))
        if copies > 1:
            X[1:].copy_(X[0].expand(copies - 1, B, V))
        entry = {"rows": B, "l2": (f"{copies} rotating copies of the input "
                                   f"({copies * B * ROW_BYTES / 2**20:.0f} MiB)" if copies > 1
                                   else "input larger than L2")}
        runs = [("sampled", wl.params)] + ([("greedy", SamplingParams())] if wl.greedy_too else [])
        for label, p in runs:
            st = states_to_tensor(wl.row_states(row0, B), dev)
            ids = torch.empty(B, dtype=torch.int32, device=dev)
            it = [0]

            def call(p=p, st=st, ids=ids):
                s.sample(X[it[0] % copies], p, st, out=ids, stream=stream)
                it[0] += 1
            for _ in range(5):
                call()
            torch.cuda.synchronize()
            reps = max(20, min(400, int(0.1 / max(B * ROW_BYTES / (peak * 1e9), 1e-6))))
            steps = []
            ms = time_device_steps(call, reps, stream, per_step=steps) / reps
            # the same calls captured in a CUDA graph and replayed: device time without
            # the host's per-call work (bindings, planning, launches)
            graph_us = None
            try:
                n_cap = 16
                graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(graph):
                    for q in range(n_cap):
                        s.sample(X[q % copies], p, st, out=ids)
                graph.replay()
                torch.cuda.synchronize()
                reps_g = max(2, reps // n_cap)
                graph_us = time_device_steps(graph.replay, reps_g, stream) / (reps_g * n_cap) * 1e3
                del graph
            except Exception as e:  # reported, never fatal
                graph_us = f"capture failed: {e}"
            s.get_timing()
            s.set_timing(True)
            time_device_steps(call, 10, stream)
            kt = s.get_timing()
            s.set_timing(False)
            gbs = B * ROW_BYTES / (ms / 1e3) / 1e9
            r = {"params": describe(p), "us_per_call": ms * 1e3, "rows_per_s": B / (ms / 1e3),
                 "us_per_call_graph": graph_us,
                 "logits_gbs": gbs, "hbm_frac": gbs / peak,
                 "per_call_us": {k2: v * 1e3 for k2, v in spread(steps).items() if k2 != "n"},
                 "select_us": kt["select_ms"] / 10 * 1e3, "merge_us": kt["merge_ms"] / 10 * 1e3,
                 "large_us": kt["large_ms"] / 10 * 1e3,
                 "select_gbs": (B * ROW_BYTES / (kt["select_ms"] / 10 / 1e3) / 1e9
                                if kt["select_ms"] > 0 else None)}
            if with_parity:
                r["parity"] = parity_counts(s, dev, xh, p, wl.row_states(row0, B),
                                            wl.row_seeds(row0, B), stream)
            entry[label] = r
        out[str(cfg)] = entry
        del X
    return out


def describe(p):
    if p.temp <= 0:
        parts = ["greedy"]
    else:
        parts = [f"temp {p.temp:g}"]
        if p.top_k > 0:
            parts.append(f"top-k {p.top_k}")
        if p.top_p < 1.0:
            parts.append(f"top-p {p.top_p:g}")
    if p.repeat_penalty != 1.0:
        parts.append(f"repeat_penalty {p.repeat_penalty:g}, last {p.repeat_last_n}")
    return ", ".join(parts)


def host_api_bench(x_row):
    """The drop-in C++ API (include/zen/sample.h) as cmd_generate calls it: one host
    row per call through zen::sample_token (libzs_sampler.so's sample_shim.cpp),
    timed by the compiled driver zeninfer_b200/bench_host_api; beside it the
    reference's own sample_token on one host thread."""
    import numpy as np
    exe = os.path.join(ROOT, "zeninfer_b200", "bench_host_api")
    if not os.path.exists(exe):
        return {"note": "zeninfer_b200/bench_host_api not built"}
    out = {"rows_per_call": 1, "path": "host row -> pinned staging -> H2D -> zs_sample -> D2H id"}
    fd, path = tempfile.mkstemp(suffix=".f32")
    os.close(fd)
    try:
        np.ascontiguousarray(x_row, dtype=np.float32).tofile(path)
        cases = {"temp 0.7, top-k 40": ("0.7", "40", "1.0", "1.0", "64", "0"),
                 "temp 0.7, top-k 40, top-p 0.9, repeat_penalty 1.1, last 64, 64-id history":
                     ("0.7", "40", "0.9", "1.1", "64", "64")}
        for name, (t, k, tp, pen, ln, hl) in cases.items():
            r = subprocess.run([exe, path, str(V), "500", t, k, tp, pen, ln, hl],
                               capture_output=True, text=True, timeout=120)
            try:
                res = json.loads(r.stdout.strip().splitlines()[-1])
            except Exception:
                res = {"error": (r.stderr or r.stdout)[-300:]}
            try:
                import oracle
                from zeninfer_b200 import SamplingParams
                if oracle.have_reference():
                    p = SamplingParams(temp=float(t), top_k=int(k), top_p=float(tp),
                                       repeat_penalty=float(pen), repeat_last_n=int(ln))
                    hist = (np.arange(int(hl), dtype=np.int64) * 997 % V).astype(np.int32)[None, :]
                    row = np.ascontiguousarray(x_row[None, :], dtype=np.float32)
                    n_ref = 10
                    t0 = time.perf_counter()
                    for i in range(n_ref):
                        oracle.reference_sample(row, p, np.array([i + 1], np.uint64),
                                                hist if int(hl) else None,
                                                np.array([int(hl)], np.int32) if int(hl) else None,
                                                nthreads=1)
                    res["reference_us_per_call"] = (time.perf_counter() - t0) / n_ref * 1e6
            except Exception as e:  # reported, never fatal
                res["reference_note"] = str(e)
            out[name] = res
    finally:
        os.unlink(path)
    return out


def shard_bench(s, dev, stream, x_dev, params, states0, rows, world, rank, steps, warmup,
                max_over_ranks, barrier):
    """Vocab-sharded mode over the same rows (N > 1), both exchanges: the whole step,
    and the partials and the merge alone, so the exchange's share is the rest."""
    import torch
    from zeninfer_b200 import Sampler, states_to_tensor
    from zeninfer_b200.sharding import VocabShardedSampler, vocab_range
    lo, n_loc = vocab_range(V, world, rank)
    x_loc = x_dev[:, lo:lo + n_loc]
    nbytes = Sampler.shard_partial_bytes(rows, V, world, params)
    res = {"rows": rows, "columns_per_rank": n_loc, "scaling": "strong",
           "block_area_bytes_per_rank": nbytes}
    part = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    for owner in (True, False):
        vs = VocabShardedSampler(s, owner=owner)
        st2 = states_to_tensor(states0, dev)
        out2 = torch.empty(rows, dtype=torch.int32, device=dev)

        def shard_step():
            vs.sample(x_loc, lo, V, params, st2, out=out2, stream=stream)

        for _ in range(warmup):
            shard_step()
        torch.cuda.synchronize()
        barrier()
        ms_sh = max_over_ranks(time_device_steps(shard_step, steps, stream) / steps)
        torch.cuda.synchronize()
        barrier()
        # the rank's own kernels alone (no collective): partials, and its merge
        ms_p = time_device_steps(lambda: s.shard_partials(x_loc, lo, V, world, params, part,
                                                          stream=stream), steps, stream) / steps
        r0, n = Sampler.shard_owner_rows(rows, world, rank) if owner else (0, rows)
        gathered = vs._slots  # the blocks of the last step, as its merge read them
        st3 = states_to_tensor(states0, dev)
        ms_m = time_device_steps(lambda: s.shard_merge(gathered, world, rows, V, params, st3,
                                                       out=out2, stream=stream, rows=(r0, n)),
                                 steps, stream) / steps
        ms_p, ms_m = max_over_ranks(ms_p), max_over_ranks(ms_m)
        res["row_owner" if owner else "all_gather"] = {
            "ms_per_step": ms_sh, "rows_per_s": rows / (ms_sh / 1e3),
            "partials_ms": ms_p, "merge_ms": ms_m,
            "exchange_and_rest_ms": max(0.0, ms_sh - ms_p - ms_m),
            "merged_rows_per_rank": n, "path": "torch.distributed (NCCL) around the C ABI"}
        barrier()
    # The C ABI's own zs_sample_sharded over an NCCL communicator of this process's
    # libnccl (asynchronous: collective timeout 0), the path a C++ caller takes.
    try:
        import ctypes as C
        import torch.distributed as dist

        class NcclUniqueId(C.Structure):
            _fields_ = [("internal", C.c_char * 128)]
        nccl = C.CDLL("libnccl.so.2")
        uid = NcclUniqueId()
        if rank == 0 and nccl.ncclGetUniqueId(C.byref(uid)) != 0:
            raise RuntimeError("ncclGetUniqueId failed")
        obj = [C.string_at(C.addressof(uid), C.sizeof(uid)) if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        C.memmove(C.addressof(uid), obj[0], C.sizeof(uid))
        comm = C.c_void_p()
        if nccl.ncclCommInitRank(C.byref(comm), world, uid, rank) != 0:
            raise RuntimeError("ncclCommInitRank failed")
        st4 = states_to_tensor(states0, dev)
        out4 = torch.empty(rows, dtype=torch.int32, device=dev)
        xl = x_loc.contiguous() if x_loc.stride(1) != 1 else x_loc

        def c_step():
            s.sample_sharded(xl, lo, V, world, params, st4, comm.value, out=out4, stream=stream)
        s.set_collective_timeout(60000)  # warm-up calls wait, bounded
        for _ in range(warmup):
            c_step()
        s.set_collective_timeout(0)  # timed calls are stream-ordered only
        torch.cuda.synchronize()
        barrier()
        ms_c = max_over_ranks(time_device_steps(c_step, steps, stream) / steps)
        torch.cuda.synchronize()
        barrier()
        res["c_abi_row_owner"] = {"ms_per_step": ms_c, "rows_per_s": rows / (ms_c / 1e3),
                                  "path": "zs_sample_sharded (NCCL send/recv + all-gather inside)"}
        s.set_collective_timeout(30000)
        nccl.ncclCommDestroy(comm)
    except Exception as e:  # reported, never fatal
        res["c_abi_note"] = str(e)
    return res


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    # ~1 ms per step: 1000 steps keep the timed region long enough (about a
    # second) for the clock sampler to see it.
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--rows", type=int, default=ROWS,
                    help="rows per GPU (default 4096, the benchmark batch; smaller only "
                         "for profiling captures)")
    ap.add_argument("--logits-file", default=None,
                    help="raw <f4 [S][V] logits written by zeninfer's `logits --out` (its rows "
                         "repeated to fill the batch) instead of the synthetic workload")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-lmhead", action="store_true", help="skip the fused lm_head timing")
    ap.add_argument("--no-fullp", action="store_true", help="skip the full-vocabulary top-p timing")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-configs", action="store_true",
                    help="skip the per-workload timings and parity counts")
    ap.add_argument("--no-parity", action="store_true",
                    help="per-workload timings without the parity counts")
    ap.add_argument("--configs", default="1,2,3,4,5",
                    help="workloads of the per-workload section (comma list, default all)")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    rows = max(1, args.rows)

    world = env_int("WORLD_SIZE", 1)
    rank = env_int("RANK", 0)
    local_rank = env_int("LOCAL_RANK", 0)

    if args.impl == "reference":
        run_reference_arm(args, rank, world)
        return

    # With several ranks, libraries (NCCL's version banner) may write to stdout; keep
    # stdout for the one JSON line and send everything else written there to stderr.
    json_out = sys.stdout
    if world > 1:
        sys.stdout.flush()
        json_out = os.fdopen(os.dup(1), "w")
        os.dup2(2, 1)

    import numpy as np
    import torch
    import torch.distributed as dist
    from zeninfer_b200 import Sampler, SamplingParams, states_to_tensor
    from zeninfer_b200 import workloads as W

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(v):
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    wl = W.WORKLOADS[WORKLOAD]
    params = wl.params
    stream = torch.cuda.current_stream()

    # Host copy of this rank's rows (distinct rows per rank), pinned for the e2e leg.
    row0 = rank * rows
    x_host = torch.empty((rows, V), dtype=torch.float32).pin_memory()
    data = "synthetic"
    if args.logits_file:
        from zeninfer_b200 import logits_io
        src = logits_io.read_logits(args.logits_file, V)
        xh = x_host.numpy()
        for r in range(rows):
            xh[r] = src[(row0 + r) % src.shape[0]]
        data = f"file {os.path.basename(args.logits_file)} ({src.shape[0]} rows, repeated)"
    else:
        W.generate(WORKLOAD, rows, row0=row0, out=x_host.numpy())
    x_dev = x_host.to(dev)
    states0 = wl.row_states(row0, rows)
    st = states_to_tensor(states0, dev)
    out = torch.empty(rows, dtype=torch.int32, device=dev)
    s = Sampler(local_rank)

    def step():
        s.sample(x_dev, params, st, out=out, stream=stream)

    for _ in range(args.warmup):
        step()
    s.check_device_status(stream)
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    try:
        props = torch.cuda.get_device_properties(dev)
        pci = (f"{props.pci_domain_id:08x}:{props.pci_bus_id:02x}:{props.pci_device_id:02x}.0")
    except Exception:
        pci = None
    clocks = ClockSampler(local_rank, pci)
    clocks.start()
    s.get_timing()  # start the per-kernel event sums and launch count afresh
    s.set_timing(True)
    step_ms = []
    ms_total = time_device_steps(step, args.steps, stream, per_step=step_ms)
    s.set_timing(False)
    kt = s.get_timing()
    clk = clocks.stop()
    torch.cuda.synchronize()
    barrier()
    s.check_device_status(stream)
    ms_step = max_over_ranks(ms_total / args.steps)
    value = world * rows / (ms_step / 1e3)

    # Roofline of the dominant kernel, the streaming select (zs_wselect_kernel
    # here), timed by CUDA events around its launches on the sampler's stream
    # during the timed steps.
    peak, peak_kind = hbm_peak()
    alg_bytes = rows * ROW_BYTES + rows * 4
    sel_ms = max_over_ranks(kt["select_ms"] / args.steps)
    merge_ms = max_over_ranks(kt["merge_ms"] / args.steps)
    achieved = alg_bytes / (sel_ms / 1e3) / 1e9
    step_gbs = alg_bytes / (ms_step / 1e3) / 1e9
    traffic = committed_traffic(rows)

    # BASELINE's five workloads at their own batch sizes (1, 256, 1024, 512, 4096 rows)
    # with the select / merge split and the parity counts of one checked call each.
    by_config = None
    if rank == 0 and world == 1 and not args.no_configs:
        only = {int(c) for c in args.configs.split(",") if c.strip()}
        by_config = config_bench(s, dev, stream, peak, with_parity=not args.no_parity, only=only)
    by_batch = {}
    if by_config:
        for b, cfgw in ((1, "1"), (256, "2")):
            if cfgw not in by_config:
                continue
            e = by_config[cfgw]["sampled"]
            by_batch[str(b)] = {k2: e[k2] for k2 in ("rows_per_s", "us_per_call", "logits_gbs",
                                                      "hbm_frac", "params")}
    by_batch[str(rows)] = {"rows_per_s": rows / (ms_step / 1e3), "us_per_call": ms_step * 1e3,
                           "logits_gbs": step_gbs, "hbm_frac": step_gbs / peak,
                           "params": "temp 0.7, top-k 50, top-p 0.9"}

    # The `logits` command's display numbers (src/main.cpp:473-503) for one row,
    # the last position's, as that command computes them: device-timed, beside the
    # restatement timed on one host thread.
    display = None
    if rank == 0 and world == 1:
        x1 = x_dev[:1]
        for _ in range(3):
            s.logits_stats(x1, 8, stream=stream)
        torch.cuda.synchronize()
        reps = 100
        ms_disp = time_device_steps(lambda: s.logits_stats(x1, 8, stream=stream), reps,
                                    stream) / reps
        display = {"rows": 1, "topn": 8, "gpu_us_per_call": ms_disp * 1e3}
        try:
            import oracle
            row = x_host[:1].numpy()
            t0 = time.perf_counter()
            for _ in range(5):
                oracle.oracle_logits_stats(row, 8)
            display["cpu_restatement_us_per_call"] = (time.perf_counter() - t0) / 5 * 1e6
        except Exception as e:  # reported, never fatal
            display["cpu_restatement_us_per_call"] = None
            display["cpu_note"] = str(e)

    # The generate loop (src/main.cpp:626-632) with history, Rng states and stop
    # flags on the device (zs_decode_step): per-step device time at 1 and 256
    # sequences with the penalty on, beside the reference's sample_token per step on
    # one host thread (host logits, the history as a std::vector).
    decode = None
    if rank == 0 and world == 1:
        pdec = SamplingParams(temp=0.7, top_k=40, top_p=0.9, repeat_penalty=1.1,
                              repeat_last_n=64)
        decode = {"params": "temp 0.7, top-k 40, top-p 0.9, repeat_penalty 1.1, last 64",
                  "history_ld": 128}
        for b in (1, 256):
            xd = x_dev[:b]
            rngd = states_to_tensor(states0[:b], dev)
            doned = torch.zeros(b, dtype=torch.int32, device=dev)
            histd = torch.zeros((b, 128), dtype=torch.int32, device=dev)
            hlend = torch.zeros(b, dtype=torch.int32, device=dev)
            outd = torch.empty(b, dtype=torch.int32, device=dev)

            def dstep(xd=xd, rngd=rngd, doned=doned, histd=histd, hlend=hlend, outd=outd):
                s.decode_step(xd, pdec, rngd, doned, -1, histd, hlend, out=outd, stream=stream)

            for _ in range(5):
                dstep()
            torch.cuda.synchronize()
            reps = 200
            msd = time_device_steps(dstep, reps, stream) / reps
            decode[f"gpu_us_per_step_b{b}"] = msd * 1e3
            decode[f"tokens_per_s_b{b}"] = b / (msd / 1e3)
            # the same steps captured once in a CUDA graph (50 per graph) and replayed:
            # no host launch gaps between the step's stream operations
            try:
                graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(graph):
                    for _ in range(50):
                        s.decode_step(xd, pdec, rngd, doned, -1, histd, hlend, out=outd)
                graph.replay()
                torch.cuda.synchronize()
                reps_g = 10
                msg = time_device_steps(graph.replay, reps_g, stream) / (reps_g * 50)
                decode[f"gpu_us_per_step_b{b}_graph"] = msg * 1e3
                del graph
            except Exception as e:  # reported, never fatal
                decode["graph_note"] = str(e)
        try:
            import oracle
            if oracle.have_reference():
                row = x_host[:1].numpy()
                hist = np.arange(64, dtype=np.int32)[None, :] * 997 % V
                n_ref = 10
                t0 = time.perf_counter()
                for i in range(n_ref):
                    oracle.reference_sample(row, pdec, np.array([i + 1], np.uint64), hist,
                                            np.array([64], np.int32), nthreads=1)
                decode["reference_us_per_step_b1"] = (time.perf_counter() - t0) / n_ref * 1e6
        except Exception as e:  # reported, never fatal
            decode["reference_note"] = str(e)

    # The lm_head fused with the sampler (zs_lmhead_sample): rmsnorm + the
    # 151,936 x 896 bf16 GEMM on the tensor cores with the shortlist selection in its
    # epilogue + merge, at 4096 and 1 rows, beside the unfused library route (cuBLAS
    # bf16 GEMM with f32 logits, then zs_sample) and the reference's own CPU lm_head
    # (rmsnorm + matvec_f32, AVX2, all host threads) + sample_token on a few rows.
    lmhead = None
    if rank == 0 and world == 1 and not args.no_lmhead:
        lmhead = lmhead_bench(s, dev, stream, peak)

    # Nucleus over the whole vocabulary (top_k = n_vocab: the shortlist is every
    # token, sorted; softmax, nucleus and draw over all of it in f64), workload 3
    # (1024 rows, -1.1 log(rank+1) + noise, temp 1.0, top-p 0.95), beside the
    # reference's sample_token with the same params on a bounded sample of rows.
    fullp = None
    if rank == 0 and world == 1 and not args.no_fullp:
        fullp = full_vocab_top_p_bench(s, dev, stream)

    # End to end through the public API with host buffers: H2D of the step's
    # logits from pinned memory, the sampler, D2H of the ids, every step.
    e2e = None
    if not args.no_e2e:
        out_host = torch.empty(rows, dtype=torch.int32).pin_memory()
        x_e2e = torch.empty_like(x_dev)

        def e2e_step():
            x_e2e.copy_(x_host, non_blocking=True)
            s.sample(x_e2e, params, st, out=out, stream=stream)
            out_host.copy_(out, non_blocking=True)

        e2e_step()
        torch.cuda.synchronize()
        barrier()
        k = max(3, min(args.steps, 5))
        t0 = time.perf_counter()
        for _ in range(k):
            e2e_step()
            torch.cuda.current_stream().synchronize()
            _ = int(out_host[0])
        e2e_ms = max_over_ranks((time.perf_counter() - t0) * 1e3 / k)
        e2e = {"value": world * rows / (e2e_ms / 1e3), "unit": UNIT,
               "h2d_bytes_per_step": rows * ROW_BYTES, "d2h_bytes_per_step": rows * 4,
               "ms_per_step": e2e_ms}
        del x_e2e

    # Vocab-sharded mode over the same rows (N > 1): partials -> exchange -> merge.
    sharded = None
    if world > 1:
        sharded = shard_bench(s, dev, stream, x_dev, params, states0, rows, world, rank,
                              args.steps, args.warmup, max_over_ranks, barrier)

    # The drop-in C++ API with one host row per call (cmd_generate's call).
    host_api = None
    if rank == 0 and world == 1 and not args.no_cpu:
        host_api = host_api_bench(W.generate(1, 1)[0])

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        try:
            import oracle
            if oracle.have_reference():
                rate, n_cpu, dt, nth = cpu_reference_rate(x_host.numpy(), params,
                                                          wl.row_seeds(row0, rows))
                cpu = {"value": rate, "unit": UNIT, "cores": nth, "kind": "reference",
                       "sample": f"{n_cpu} rows of this batch ({dt:.1f} s), zen::sample_token "
                                 f"(src/sample.cpp compiled unchanged) on {nth} threads"}
        except Exception as e:  # reported, never fatal
            cpu = {"value": None, "unit": UNIT, "cores": None, "kind": "reference",
                   "sample": f"failed: {e}"}

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f32 (f64 shortlist softmax)", "data": data,
            "config": {"workload": f"{rows} x 151936 f32 logits per GPU (workload 5: N(0,2.5^2)"
                                   " + offset + 8 peaks), temp 0.7, top-k 50, top-p 0.9",
                       "rows_per_gpu": rows, "vocab": V, "parallelism": f"row-split x{world}",
                       "l2": "inputs (2.49 GB per GPU) larger than L2"},
            "logits_gbs": step_gbs, "hbm_frac": step_gbs / peak,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": traffic,
                         "peak_source": f"hbm_gbs, of {peak_kind}",
                         "kernel": "zs_wselect_kernel",
                         "kernel_ms_per_step": sel_ms, "merge_ms_per_step": merge_ms,
                         "algorithmic_bytes_per_launch": alg_bytes},
            "per_step_ms": spread(step_ms),
            "by_batch": by_batch,
            "clocks": clk,
            "e2e": e2e,
            "gpu_launches": kt["launches"],
            "gpu_launches_by_kernel": {"select": kt["select_launches"],
                                       "merge": kt["merge_launches"],
                                       "large": kt["large_launches"]},
            "cpu_baseline": cpu,
        }
        if by_config:
            line["by_config"] = by_config
        if sharded:
            line["vocab_sharded"] = sharded
        if host_api:
            line["host_api_b1"] = host_api
        if display:
            line["logits_display"] = display
        if decode:
            line["decode_loop"] = decode
        if lmhead:
            line["lmhead_fused"] = lmhead
        if fullp:
            line["full_vocab_top_p"] = fullp
        print(json.dumps(line), file=json_out, flush=True)

    s.close()
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
