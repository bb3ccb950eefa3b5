#!/usr/bin/env python
"""Benchmark of the int8 weight-only dequant-matmul path on B200.

One step = one pass of the hot path over one batch of synthetic input: one
call of popcornDequantizeMatmul_i8f32 (popcorn src/quantize.cu:86-112) on the
headline workload, the memory-bound decode GEMV M=1, K=4096, N=4096. With
--gpus N > 1 the weight rows are N-sharded (column-parallel) across ranks and
every step ends with an NCCL all-gather of the output shards, so the whole
job still computes the full 4096-wide output per step (strong scaling).

Timing: W eager warm-up steps, then an untimed soak of CUDA-graph replays
(clocks settle, NVML samples them), then EXACTLY K steps replayed from one
CUDA graph, bracketed by barrier + synchronize, timed with CUDA events on the
launching stream; the max over ranks is reported. Weights rotate over a pool
of independent weight sets larger than 2x L2, so every step streams its
weights from HBM.

Arms:
  (default)          this library, through its C ABI (ctypes on the in-tree .so)
  --impl reference   popcorn's own CPU loop (test/test_quantize.cu:24-41,
                     compiled from the reference sources into oracle/_ref) on
                     all host cores of rank 0; also reports popcorn's own CUDA
                     kernel rebuilt for sm_100a as an extra key.
"""
import argparse
import json
import math
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "W8 dequant-matmul: int8-weight GB/s at M=1; TFLOPS at M=2048 (1/2/4/8 B200)"

# Workloads: the headline plus the other single-GPU configurations reported as
# extra keys. bytes = int8 weight bytes per step; flops = 2*M*N*K.
WORKLOADS = {
    "decode": dict(M=1, K=4096, N=4096, unit="GB/s", bound="hbm"),
    "skinny": dict(M=32, K=4096, N=11008, unit="GB/s", bound="hbm"),
    "prefill": dict(M=2048, K=4096, N=4096, unit="TFLOP/s", bound="tensor"),
    # Per-group int8 (popcornDequantizeMatmulGrouped_i8f32), decode size, group 128:
    # algorithmic bytes = codes + group scales.
    "grouped_decode": dict(M=1, K=4096, N=4096, unit="GB/s", bound="hbm", group_size=128),
    # Int4 packed asymmetric (popcornDequantizeMatmulGrouped_i4f32), decode size,
    # group 128: algorithmic bytes = packed codes + group scales and zero points.
    "int4_decode": dict(M=1, K=4096, N=4096, unit="GB/s", bound="hbm", group_size=128, bits=4),
    # The same two formats at prefill size (tensor cores, group factors in the converters).
    "grouped_prefill": dict(M=2048, K=4096, N=4096, unit="TFLOP/s", bound="tensor", group_size=128),
    "int4_prefill": dict(M=2048, K=4096, N=4096, unit="TFLOP/s", bound="tensor", group_size=128, bits=4),
    # Front of a gated MLP at decode size (7B shapes): RMSNorm -> gate and up
    # projections 4096 -> 11008 -> SiLU(gate) * up, in one fused call
    # (popcornRMSNormDequantizeMatmulSiluMul_i8f32); algorithmic bytes = both
    # int8 weight matrices. The unfused sequence is timed beside it.
    "mlp_decode": dict(M=1, K=4096, N=11008, unit="GB/s", bound="hbm", mlp=True),
    # The weight-side kernels around the matmul at the decode layer's size:
    # popcornQuantize_f32i8 (bytes 5*N*K + 4*N: read f32, write codes and
    # scales) and popcornDequantize_i8f32 (bytes N*K + 4*N + 4*N*K: read
    # codes and scales, write f32).
    "quantize": dict(M=0, K=4096, N=4096, unit="GB/s", bound="hbm", op="quantize"),
    "dequantize": dict(M=0, K=4096, N=4096, unit="GB/s", bound="hbm", op="dequantize"),
    "dequantize_bf16": dict(M=0, K=4096, N=4096, unit="GB/s", bound="hbm", op="dequantize", out_bytes=2),
    # The stack's qkv projection at 128 activation rows (4096 -> 12288): the
    # int8 tensor path on CTA pairs; FLOPs = 2*M*N*K.
    "qkv_m128": dict(M=128, K=4096, N=12288, unit="TFLOP/s", bound="tensor"),
}

# Per-launch DRAM traffic (dram__bytes_read.sum + dram__bytes_write.sum) of
# the dominant kernel from one ncu capture of that workload; the command that
# produced each figure is in the profiles/ summary named beside it. The
# quantizer and the expand kernels are left out: most of what they write is
# still in L2 when a captured launch ends, so DRAM writes under-count it
# (their profiles give the figures).
NCU_TRAFFIC = {
    "decode": 16826624,    # profiles/gemv_mma_decode_m1_k4096_n4096.md
    "skinny": 45440256,    # profiles/tc_i8_skinny_m32_k4096_n11008.md
    "prefill": 35509504,   # profiles/tc_gemm_pair_prefill_m2048_k4096_n4096.md
    "grouped_decode": 17352704,  # profiles/grouped_mma_decode_m1_k4096_n4096_g128.md
    "int4_decode": 9487360,      # profiles/i4_mma_decode_m1_k4096_n4096_g128.md
    "mlp_decode": 94391296,      # profiles/fused_xs_mlp_decode_m1_k4096_n11008.md
    "qkv_m128": 51826176,        # profiles/tc_i8_pair_m128_k4096_n12288.md
}


def parse_args():
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=2000)
    p.add_argument("--warmup", type=int, default=10)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--workload", choices=sorted(WORKLOADS), default="decode")
    p.add_argument("--extras", default="skinny,prefill,grouped_decode,int4_decode,grouped_prefill,int4_prefill,"
                                       "mlp_decode,quantize,dequantize,dequantize_bf16,qkv_m128",
                   help="comma-separated extra single-GPU workloads reported beside the headline (N=1 only)")
    p.add_argument("--stack", default="1,128",
                   help="M values of the 32-layer 7B-shaped linear stack timed at every N ('none' to skip)")
    p.add_argument("--stack-layers", type=int, default=32)
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--soak-s", type=float, default=0.6)
    return p.parse_args()


# ---------------------------------------------------------------------------
# Environment helpers
# ---------------------------------------------------------------------------
def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def measured_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return dict(hbm=float(d["hbm_gbs"]), tc=float(d["bf16_tflops"]),
                    tc_sustained=float(d.get("bf16_tflops_sustained", d["bf16_tflops"])), source="measured")
    except (OSError, KeyError, ValueError):
        return dict(hbm=6650.0, tc=1590.0, tc_sustained=1400.0, source="fallback")


def host_threads():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


class ClockSampler:
    """NVML sampling of SM clock and throttle reasons in a background thread."""

    REASONS = {
        "gpu_idle": 0x1, "applications_clocks_setting": 0x2, "sw_power_cap": 0x4, "hw_slowdown": 0x8,
        "sync_boost": 0x10, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40,
        "hw_power_brake_slowdown": 0x80, "display_clock_setting": 0x100,
    }

    def __init__(self, device, period_s=0.01):
        self.samples = []  # (t, sm_mhz, reasons_mask)
        self.period = period_s
        self.ok = False
        self.max_mhz = None
        try:
            import pynvml
            import torch

            pynvml.nvmlInit()
            self.nvml = pynvml
            # Map the CUDA device to its NVML handle by PCI address (NVML does
            # not see CUDA_VISIBLE_DEVICES renumbering).
            p = torch.cuda.get_device_properties(device)
            bus = f"{p.pci_domain_id:08x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"
            self.h = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception:  # noqa: BLE001 - clocks are reported as unavailable
            self.ok = False
        self._stop = threading.Event()
        self._t = None

    def _run(self):
        while not self._stop.is_set():
            try:
                mhz = self.nvml.nvmlDeviceGetClockInfo(self.h, self.nvml.NVML_CLOCK_SM)
                rs = self.nvml.nvmlDeviceGetCurrentClocksThrottleReasons(self.h)
                self.samples.append((time.perf_counter(), mhz, rs))
            except Exception:  # noqa: BLE001
                pass
            time.sleep(self.period)

    def start(self):
        if self.ok:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()

    def stop(self):
        if self._t is not None:
            self._stop.set()
            self._t.join()

    def summary(self, t0, t1, t_timed0, t_timed1):
        if not self.ok:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvml unavailable"]}
        window = [s for s in self.samples if t0 <= s[0] <= t1]
        in_timed = [s for s in window if t_timed0 <= s[0] <= t_timed1]
        loaded = [s for s in window if not (s[2] & self.REASONS["gpu_idle"])] or window
        mhz = statistics.median([s[1] for s in loaded]) if loaded else None
        mask = 0
        for s in loaded:
            mask |= s[2]
        reasons = [k for k, v in self.REASONS.items() if mask & v and k != "gpu_idle"]
        return {"sm_mhz": mhz, "sm_max_mhz": self.max_mhz, "reasons": reasons,
                "samples": len(loaded), "samples_in_timed_region": len(in_timed),
                "window": "soak+timed (same graph replays)"}


# ---------------------------------------------------------------------------
# Our arm
# ---------------------------------------------------------------------------
class Setup:
    """Device-resident synthetic inputs for one workload on one rank."""

    def __init__(self, torch, pc, wl, rank, world, device, pool_bytes):
        self.torch = torch
        self.pc = pc
        M, K, N = wl["M"], wl["K"], wl["N"]
        assert N % world == 0, "N must divide evenly across ranks"
        self.M, self.K, self.N = M, K, N
        self.Nl = N // world
        self.world = world
        self.gs = wl.get("group_size")
        self.bits = wl.get("bits", 8)
        per_set = self.Nl * K * self.bits // 8 + (M * K * 4 if wl["bound"] == "tensor" else 0)
        self.sets = max(2, math.ceil(pool_bytes / per_set))
        if wl["bound"] == "tensor":
            self.sets = min(self.sets, 4)
        # Every rank draws the same full matrices and inputs (seeds do not
        # depend on the rank) and keeps its row shard, so the N-sharded job
        # computes exactly what one GPU computes over the full weights.
        g = torch.Generator(device=device)
        lo, hi = rank * self.Nl, (rank + 1) * self.Nl
        self.q, self.s, self.z, self.x, self.out = [], [], [], [], []
        self.q_full = self.s_full = None
        for i in range(self.sets):
            # W ~ N(0, 0.02) f32 quantized (per row, per group or int4 per
            # group) by this library's quantizer.
            g.manual_seed(1234 + i)
            w = torch.randn((N, K), generator=g, device=device) * 0.02
            if self.bits == 4:
                q, s, z = pc.quantize_grouped_i4(w, self.gs)
                self.z.append(z[lo:hi].contiguous())
            else:
                q, s = pc.quantize_grouped(w, self.gs) if self.gs else pc.quantize(w)
            del w
            if i == 0 and world > 1 and not self.gs:
                self.q_full, self.s_full = q, s
            self.q.append(q[lo:hi].contiguous())
            self.s.append(s[lo:hi].contiguous())
            if wl["bound"] == "tensor" or i == 0:
                g.manual_seed(99 + i)
                self.x.append(torch.randn((M, K), generator=g, device=device))
            self.out.append(torch.empty((M, self.Nl), dtype=torch.float32, device=device))
        self.gathered = torch.empty((world * M * self.Nl,), dtype=torch.float32, device=device)
        torch.cuda.synchronize()
        self.lib = pc.load_library()
        # Multi-GPU decode: the all-gather is fused into the GEMV (tagged
        # NVLink peer stores); other shapes use an NCCL all-gather.
        self.fused = None
        if world > 1 and M <= 4:
            from popcorn_b200.tp import PeerGroup

            self.fused = PeerGroup(M, N, device)
            self.n_offset = rank * self.Nl
            self.full = torch.empty((M, N), dtype=torch.float32, device=device)

    def xi(self, i):
        return self.x[i % len(self.x)]

    def step(self, i, stream_handle, group=None):
        j = i % self.sets
        x = self.xi(i)
        if self.fused is not None:
            st = self.fused.all_gather(self.full, x, self.q[j], self.s[j], self.n_offset, stream_handle)
            if st != 0:
                raise RuntimeError(f"popcornDequantizeMatmulAllGather_i8f32 failed: {st}")
            return
        if self.bits == 4:
            st = self.lib.popcornDequantizeMatmulGrouped_i4f32(self.out[j].data_ptr(), x.data_ptr(),
                                                               self.q[j].data_ptr(), self.s[j].data_ptr(),
                                                               self.z[j].data_ptr(), self.M, self.Nl, self.K, self.gs,
                                                               stream_handle)
        elif self.gs:
            st = self.lib.popcornDequantizeMatmulGrouped_i8f32(self.out[j].data_ptr(), x.data_ptr(),
                                                               self.q[j].data_ptr(), self.s[j].data_ptr(), self.M,
                                                               self.Nl, self.K, self.gs, stream_handle)
        else:
            st = self.lib.popcornDequantizeMatmul_i8f32(self.out[j].data_ptr(), x.data_ptr(), self.q[j].data_ptr(),
                                                        self.s[j].data_ptr(), self.M, self.Nl, self.K, stream_handle)
        if st != 0:
            raise RuntimeError(f"dequant-matmul call failed: {st} "
                               f"{self.lib.popcornGetLastCudaErrorString().decode()}")
        if self.world > 1:
            self.torch.distributed.all_gather_into_tensor(self.gathered, self.out[j].view(-1), group=group)

    def tp_parity(self, stream_handle):
        """After one sharded step on weight set 0: the gathered [M, N] output
        against a single-GPU popcornDequantizeMatmul_i8f32 over the full
        weights on this rank (bit-exact expected: same per-row arithmetic)."""
        torch = self.torch
        self.step(0, stream_handle)
        if self.fused is not None:
            got = self.full.clone()
        else:
            parts = self.gathered.view(self.world, self.M, self.Nl)
            got = torch.cat([parts[r] for r in range(self.world)], dim=1)
        ref = torch.empty((self.M, self.N), dtype=torch.float32, device=got.device)
        st = self.lib.popcornDequantizeMatmul_i8f32(ref.data_ptr(), self.x[0].data_ptr(), self.q_full.data_ptr(),
                                                    self.s_full.data_ptr(), self.M, self.N, self.K, stream_handle)
        if st != 0:
            raise RuntimeError(f"single-GPU reference call failed: {st}")
        torch.cuda.synchronize()
        err = float((got.double() - ref.double()).abs().max() / ref.double().abs().max())
        bitexact = bool(torch.equal(got.view(torch.int32), ref.view(torch.int32)))
        return {"what": "gathered output vs one GPU over the full weights (same x, set 0)",
                "max_err": err, "bitexact": bitexact, "ok": bitexact}

    def grouped_tensor(self):
        """Per-group formats take the tensor-core path (prologue + GEMM) above
        four activation rows and 2^27 multiply-adds."""
        return bool(self.gs) and self.M > 4 and self.M * self.Nl * self.K >= (1 << 27) and self.gs % 32 == 0

    def launches_per_step(self):
        if self.fused is not None:
            return 1
        if self.gs:
            return 2 if self.grouped_tensor() else 1
        return self.pc.launch_count(self.x[0].data_ptr(), self.q[0].data_ptr(), self.M, self.Nl, self.K)

    def path(self):
        if self.gs:
            fmt = "int4" if self.bits == 4 else "grouped"
            sms = self.torch.cuda.get_device_properties(self.x[0].device).multi_processor_count
            if self.bits != 4 and self.M == 1 and staged_mma_grouped(self.K, self.Nl, self.gs, sms):
                return f"grouped_f32 (group {self.gs}, staged rows, mma.sync s8)"
            if self.bits == 4 and self.M == 1 and staged_mma_i4(self.K, self.Nl, self.gs, sms):
                return f"int4 (group {self.gs}, staged rows, mma.sync u8)"
            return f"{fmt}_{'tensor_f16' if self.grouped_tensor() else 'f32'} (group {self.gs})"
        path = self.pc.select_path(self.x[0].data_ptr(), self.q[0].data_ptr(), self.M, self.Nl, self.K)
        if path == self.pc.PATH_TENSOR_F16 and self.M <= 128 and self.K <= 65536:
            return "tensor_i8 (activations as two int8 digits)"
        sms = self.torch.cuda.get_device_properties(self.x[0].device).multi_processor_count
        if path == self.pc.PATH_SIMT_F32 and self.M == 1 and staged_mma(self.K, self.Nl, sms):
            return "simt_f32 (staged rows, mma.sync s8)"
        return self.pc.PATH_NAMES[path]


class MlpSetup:
    """RMSNorm -> gate and up projections -> SiLU(gate) * up at decode size,
    either as one fused call or as the unfused sequence (torch RMSNorm, two
    popcornDequantizeMatmul_i8f32 calls, torch SiLU and multiply)."""

    EPS = 1e-5

    def __init__(self, torch, pc, wl, device, pool_bytes, fused=True):
        M, K, N = wl["M"], wl["K"], wl["N"]
        self.torch, self.M, self.K, self.N, self.fused = torch, M, K, N, fused
        self.sets = max(2, math.ceil(pool_bytes / (2 * N * K)))
        g = torch.Generator(device=device)
        g.manual_seed(4321)
        self.qg, self.sg, self.qu, self.su = [], [], [], []
        for _ in range(self.sets):
            for qs, ss in ((self.qg, self.sg), (self.qu, self.su)):
                w = torch.randn((N, K), generator=g, device=device) * 0.02
                q, sc = pc.quantize(w)
                del w
                qs.append(q)
                ss.append(sc)
        self.x = torch.randn((M, K), generator=g, device=device)
        self.nw = 1.0 + 0.1 * torch.randn((K,), generator=g, device=device)
        self.out = torch.empty((M, N), dtype=torch.float32, device=device)
        self.u = torch.empty_like(self.out)
        self.xn = torch.empty_like(self.x)
        self.lib = pc.load_library()
        self.Nl = N
        torch.cuda.synchronize()

    def launches_per_step(self):
        return 1 if self.fused else 2

    def step(self, i, stream_handle, group=None):
        j = i % self.sets
        lib, torch = self.lib, self.torch
        if self.fused:
            st = lib.popcornRMSNormDequantizeMatmulSiluMul_i8f32(
                self.out.data_ptr(), self.x.data_ptr(), self.nw.data_ptr(), self.EPS, self.qg[j].data_ptr(),
                self.sg[j].data_ptr(), self.qu[j].data_ptr(), self.su[j].data_ptr(), self.M, self.N, self.K,
                stream_handle)
            if st != 0:
                raise RuntimeError(f"fused MLP call failed: {st}")
            return
        torch.mul(self.x * torch.rsqrt(self.x.pow(2).mean(-1, keepdim=True) + self.EPS), self.nw, out=self.xn)
        for dst, q, sc in ((self.out, self.qg[j], self.sg[j]), (self.u, self.qu[j], self.su[j])):
            st = lib.popcornDequantizeMatmul_i8f32(dst.data_ptr(), self.xn.data_ptr(), q.data_ptr(), sc.data_ptr(),
                                                   self.M, self.N, self.K, stream_handle)
            if st != 0:
                raise RuntimeError(f"dequant-matmul call failed: {st}")
        torch.mul(torch.nn.functional.silu(self.out), self.u, out=self.out)

    def path(self):
        return "fused rmsnorm + gate/up + silu*mul" if self.fused else "unfused sequence"


LEAD_IN_CYCLES = 2_000_000  # ~1 ms of GPU time at 1.9 GHz


def lead_in(torch):
    """Keep the stream busy (a spin kernel of ~1 ms) while the host enqueues
    the start event, the graph and the end event, so the events bracket the K
    steps themselves and not the host's submission latency."""
    torch.cuda._sleep(LEAD_IN_CYCLES)


class OpSetup:
    """popcornQuantize_f32i8 or popcornDequantize_i8f32 on [N, K], rotating
    over enough independent buffers that every step reads and writes HBM."""

    def __init__(self, torch, pc, wl, device, pool_bytes):
        N, K = wl["N"], wl["K"]
        self.op, self.N, self.K = wl["op"], N, K
        self.bf16 = wl.get("out_bytes", 4) == 2
        self.sets = max(2, math.ceil(pool_bytes / weight_bytes(wl)))
        g = torch.Generator(device=device)
        g.manual_seed(555)
        self.w, self.q, self.s = [], [], []
        for _ in range(self.sets):
            w = torch.randn((N, K), generator=g, device=device) * 0.02
            q, sc = pc.quantize(w)
            self.w.append(w.to(torch.bfloat16) if self.bf16 else w)
            self.q.append(q)
            self.s.append(sc)
        self.lib = pc.load_library()
        self.Nl = N
        torch.cuda.synchronize()

    def launches_per_step(self):
        return 1

    def step(self, i, stream_handle, group=None):
        j = i % self.sets
        if self.op == "quantize":
            st = self.lib.popcornQuantize_f32i8(self.q[j].data_ptr(), self.s[j].data_ptr(), self.w[j].data_ptr(),
                                                self.N, self.K, stream_handle)
        else:
            fn = self.lib.popcornDequantize_i8bf16 if self.bf16 else self.lib.popcornDequantize_i8f32
            st = fn(self.w[j].data_ptr(), self.q[j].data_ptr(), self.s[j].data_ptr(), self.N, self.K, stream_handle)
        if st != 0:
            raise RuntimeError(f"{self.op} call failed: {st}")

    def path(self):
        if self.op == "quantize":
            return "popcornQuantize_f32i8"
        return "popcornDequantize_i8bf16 (bf16 out)" if self.bf16 else "popcornDequantize_i8f32 (f32 out)"


def time_graph(torch, setup, steps, warmup, soak_s, sampler, dist_on):
    """Warm up, soak, then time exactly `steps` steps from one CUDA graph."""
    stream = torch.cuda.Stream()
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        for i in range(warmup):
            setup.step(i, stream.cuda_stream)
    stream.synchronize()

    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for i in range(steps):
            setup.step(i, stream.cuda_stream)
    torch.cuda.synchronize()

    t_soak0 = time.perf_counter()
    with torch.cuda.stream(stream):
        graph.replay()
    stream.synchronize()
    once = time.perf_counter() - t_soak0
    reps = max(1, int(soak_s / max(once, 1e-6)))
    if dist_on:
        # Every rank must replay the same number of graphs (each holds the
        # same sequence of NCCL collectives), so agree on the count.
        t = torch.tensor([reps], dtype=torch.int64, device=torch.device("cuda", torch.cuda.current_device()))
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        reps = int(t.item())
    with torch.cuda.stream(stream):
        for _ in range(reps):
            graph.replay()
    stream.synchronize()

    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    if dist_on:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    t_timed0 = time.perf_counter()
    with torch.cuda.stream(stream):
        lead_in(torch)
        start.record(stream)
        graph.replay()
        end.record(stream)
    torch.cuda.synchronize()
    t_timed1 = time.perf_counter()
    if dist_on:
        torch.distributed.barrier()
    ms = start.elapsed_time(end)
    clocks = sampler.summary(t_soak0, t_timed1, t_timed0, t_timed1) if sampler else None
    del graph
    return ms, clocks


def _cudart():
    """The CUDA runtime torch has loaded (for per-step copies without torch's
    dispatch overhead)."""
    import ctypes

    rt = ctypes.CDLL("libcudart.so.12")
    rt.cudaMemcpyAsync.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int, ctypes.c_void_p]
    rt.cudaMemcpyAsync.restype = ctypes.c_int
    rt.cudaStreamSynchronize.argtypes = [ctypes.c_void_p]
    rt.cudaStreamSynchronize.restype = ctypes.c_int
    return rt


def time_e2e(torch, setup, steps, warmup, dist_on):
    """Same steps through the C ABI with host buffers, every step: pinned H2D
    of x (cudaMemcpyAsync), the library call, pinned D2H of the (gathered)
    result, and a stream synchronize before the host reads it."""
    M, K, N = setup.M, setup.K, setup.N
    stream = torch.cuda.Stream()
    sh = stream.cuda_stream
    rt = _cudart()
    h2d, d2h = 1, 2  # cudaMemcpyHostToDevice, cudaMemcpyDeviceToHost
    x_host = torch.randn((M, K)).pin_memory()
    y_host = torch.empty((M * N,), dtype=torch.float32).pin_memory()
    x_dev = torch.empty((M, K), dtype=torch.float32, device=setup.x[0].device)
    xb, yb = M * K * 4, M * N * 4
    lib = setup.lib

    def one(i):
        j = i % setup.sets
        if rt.cudaMemcpyAsync(x_dev.data_ptr(), x_host.data_ptr(), xb, h2d, sh) != 0:
            raise RuntimeError("H2D copy failed")
        if setup.fused is not None:
            st = setup.fused.all_gather(setup.full, x_dev, setup.q[j], setup.s[j], setup.n_offset, sh)
            if st != 0:
                raise RuntimeError("popcornDequantizeMatmulAllGather_i8f32 failed in e2e loop")
            src = setup.full
        else:
            st = lib.popcornDequantizeMatmul_i8f32(setup.out[j].data_ptr(), x_dev.data_ptr(), setup.q[j].data_ptr(),
                                                   setup.s[j].data_ptr(), M, setup.Nl, K, sh)
            if st != 0:
                raise RuntimeError("popcornDequantizeMatmul_i8f32 failed in e2e loop")
            src = setup.out[j]
            if setup.world > 1:
                torch.distributed.all_gather_into_tensor(setup.gathered, setup.out[j].view(-1))
                src = setup.gathered
        if rt.cudaMemcpyAsync(y_host.data_ptr(), src.data_ptr(), yb, d2h, sh) != 0:
            raise RuntimeError("D2H copy failed")
        if rt.cudaStreamSynchronize(sh) != 0:
            raise RuntimeError("stream synchronize failed")

    with torch.cuda.stream(stream):
        for i in range(warmup):
            one(i)
        if dist_on:
            torch.distributed.barrier()
        torch.cuda.synchronize()
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        start.record(stream)
        for i in range(steps):
            one(i)
        end.record(stream)
        torch.cuda.synchronize()
    if dist_on:
        torch.distributed.barrier()
    ms = start.elapsed_time(end)
    return ms, xb, yb


def staged_mma(K, N, sms):
    """Whether an M = 1 per-channel call runs the staged decode kernel with
    mma.sync: K % 32 == 0, 32 <= K <= 8192, each SM's rows (at most 64)
    within 115,648 bytes at a pitch of K + 16, and at most 20 MMAs per warp
    (16-row groups x k-steps per warp)."""
    if K % 32 or not 32 <= K <= 8192 or N < 1:
        return False
    rows = -(-N // min(sms, N))
    per_warp = -(-(K // 32) // 16)
    return rows <= 64 and rows * max(K + 16, 128) <= 115648 and -(-rows // 16) * per_warp <= 20


def staged_mma_grouped(K, N, gs, sms):
    """Whether an M = 1 per-group int8 call runs the staged mma.sync decode:
    K of 1024, 2048 or 4096, group_size % 32 == 0 with a warp's K / 16
    columns holding whole groups or lying in one (at K = 4096 groups of at
    least 128; at K = 2048 at least 64), each SM's rows (at most 64) within
    115,648 bytes at a pitch of K + 16, and at most 20 MMAs per warp."""
    if K not in (1024, 2048, 4096) or gs % 32 or N < 1:
        return False
    span = K // 16
    if span % gs and gs % span:
        return False
    gsteps = K // 512 if gs >= span else gs // 32
    if (K == 4096 and gsteps < 4) or (K == 2048 and gsteps < 2):
        return False
    rows = -(-N // min(sms, N))
    return rows <= 64 and rows * (K + 16) <= 115648 and -(-rows // 16) * (K // 512) <= 20


def staged_mma_i4(K, N, gs, sms):
    """Whether an M = 1 int4 call runs the staged mma.sync decode: K of 1024,
    2048 or 4096, group_size a multiple of 64 (of 128 at K = 4096; not 64 at
    K = 2048) with a warp's K / 16 columns holding whole groups or lying in
    one, K / group_size % 4 == 0, each SM's rows (at most 64) within 115,648
    bytes of codes at a pitch of K / 2 + 16, scales, zero points and 4 K
    bytes of converted activations, and at most 20 MMAs per warp."""
    if K not in (1024, 2048, 4096) or gs % 64 or (K // gs) % 4 or N < 1:
        return False
    span = K // 16
    if span % gs and gs % span:
        return False
    gsteps = K // 512 if gs >= span else gs // 32
    if (K == 4096 and gsteps < 4) or (K == 2048 and gsteps < 4):
        return False
    rows = -(-N // min(sms, N))
    smem = rows * (K // 2 + 16 + 8 * (K // gs + 4)) + 4 * K
    return rows <= 64 and smem <= 115648 and -(-rows // 16) * (K // 512) <= 20


def compute_dtype(path, M, K, grouped):
    """Arithmetic of the path a workload takes. The staged M = 1 decode
    (per channel, K % 32 == 0, K <= 8192, rows fitting): x as 30-bit fixed point per warp in
    four signed base-256 digits, mma.sync s8 x s8 -> s32 column sums, exact
    partials in f64. Other CUDA-core cases at M = 1: each thread's
    16-column slice of x as 30-bit fixed point, int8 codes, exact dp2a int32
    sums, then f32; otherwise f32. Tensor cores: per-channel int8 weights
    with M <= 128 (K <= 65536) run tcgen05 kind::i8 on activations held as
    16-bit fixed point in two int8 digits, everything else f16 x f16 with
    f32 accumulation."""
    if "mma.sync u8" in path:
        return "s30 fixed-point as 4 s8 digits x u4 codes (mma.sync u8.s8) -> s32/f64"
    if "mma.sync" in path:
        return "s30 fixed-point as 4 s8 digits x s8 (mma.sync) -> s32/f64"
    if "tensor" not in path:
        if M == 1 and not grouped:
            return "s30 fixed-point x s8 (dp2a) -> s32/f32"
        return "f32"
    if not grouped and M <= 128 and K <= 65536:
        return "s8x(2 s8 digits)->s32"
    return "f16xf16->f32"


def max_over_ranks(torch, value, dist_on, device):
    if not dist_on:
        return value
    t = torch.tensor([value], dtype=torch.float64, device=device)
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


def weight_bytes(wl):
    """Algorithmic bytes of one call: the codes (int8, or int4 packed two per
    byte), plus the scales (and int4 zero points) of a grouped layout; for
    the quantizer and dequantizer every byte read and written."""
    op = wl.get("op")
    if op == "quantize":
        return 5 * wl["N"] * wl["K"] + 4 * wl["N"]
    if op == "dequantize":
        return wl["N"] * wl["K"] + 4 * wl["N"] + wl.get("out_bytes", 4) * wl["N"] * wl["K"]
    if wl.get("mlp"):
        return 2 * wl["N"] * wl["K"]
    gs = wl.get("group_size")
    bits = wl.get("bits", 8)
    params = (4 if bits == 8 else 8) * wl["N"] * (wl["K"] // gs) if gs else 0
    return wl["N"] * wl["K"] * bits // 8 + params


def throughput(wl, ms_per_step):
    if wl["unit"] == "GB/s":
        return weight_bytes(wl) / (ms_per_step * 1e-3) / 1e9
    return 2.0 * wl["M"] * wl["N"] * wl["K"] / (ms_per_step * 1e-3) / 1e12


def roofline(wl, ms_per_launch, peaks, workload_name):
    if wl["bound"] == "hbm":
        achieved = weight_bytes(wl) / (ms_per_launch * 1e-3) / 1e9
        peak, unit = peaks["hbm"], "GB/s"
    else:
        achieved = 2.0 * wl["M"] * wl["N"] * wl["K"] / (ms_per_launch * 1e-3) / 1e12
        peak, unit = peaks["tc"], "TFLOP/s"
    return {"bound": wl["bound"], "achieved": round(achieved, 2), "peak": peak, "unit": unit,
            "frac": round(achieved / peak, 4), "peak_source": peaks["source"],
            "traffic": NCU_TRAFFIC.get(workload_name)}


def _time_host(run, budget_s):
    """Repeat `run` for about `budget_s` seconds of wall-clock (at least once,
    at most 200 times, after one untimed call); returns (reps, seconds per call)."""
    t0 = time.perf_counter()
    run()
    one = time.perf_counter() - t0
    reps = max(1, min(200, int(budget_s / max(one, 1e-6))))
    t0 = time.perf_counter()
    for _ in range(reps):
        run()
    return reps, (time.perf_counter() - t0) / reps


def cpu_baseline(torch, setup, wl):
    """popcorn's own CPU loop (oracle/_ref) on all host threads, bounded
    sample, plus the same loop on one core."""
    import oracle

    threads = host_threads()
    M, K, N = wl["M"], wl["K"], wl["N"]
    use_ref = oracle.have_ref_loops()
    kind = "reference" if use_ref else "port"
    x = setup.x[0][:M].cpu().numpy()
    q = setup.q[0].cpu().numpy()
    s = setup.s[0].cpu().numpy()
    rows = q.shape[0]

    def run(nt):
        if use_ref:
            oracle.ref_dequant_matmul(x, q, s, threads=nt)
        else:
            oracle.dequant_matmul(x, q, s, threads=nt)

    def rate(dt):
        if wl["unit"] == "GB/s":
            return rows * K / dt / 1e9
        return 2.0 * M * rows * K / dt / 1e12

    reps, dt = _time_host(lambda: run(threads), 2.0)
    reps1, dt1 = _time_host(lambda: run(1), 1.0)
    return {"value": round(rate(dt), 4), "unit": wl["unit"], "cores": threads, "kind": kind,
            "sample": f"{reps} full calls M={M} K={K} N={rows} (one weight set), {dt*1e3:.2f} ms each, "
                      f"wall-clock, {threads} threads",
            "single_core": {"value": round(rate(dt1), 4), "unit": wl["unit"], "cores": 1,
                            "sample": f"{reps1} full calls, {dt1*1e3:.2f} ms each, one thread"}}


def stack_shards(torch, pc, dims, layers, rank, world, device, seed, keep_full=0):
    """This rank's shards of `layers` random layers, and the full quantized
    weights of the first `keep_full` layers.

    Every matrix is drawn whole from a seed of its own (layer, part) that does
    not depend on the rank (W ~ N(0, 0.02) f32, quantized per row by
    popcornQuantize_f32i8), so the ranks' shards are slices of one model:
    rows of qkv, gate and up (column-parallel), columns of o and down
    (row-parallel, with the full per-row scale)."""
    from popcorn_b200.tp import STACK_PARTS, shard_stack_layer, stack_part_shape

    g = torch.Generator(device=device)
    out, full_layers = [], []
    for li in range(layers):
        full = {}
        for pi, part in enumerate(STACK_PARTS):
            N, K = stack_part_shape(dims, part)
            g.manual_seed(seed + 16 * li + pi)
            w = torch.randn((N, K), generator=g, device=device) * 0.02
            full[part] = pc.quantize(w)
            del w
        out.append(shard_stack_layer(full, rank, world))
        if li < keep_full:
            full_layers.append(full)
        del full
    return out, full_layers


def stack_reference(torch, pc, full_layers, x, world, dims):
    """The same layers unsharded on this GPU (single-GPU library calls),
    wired as the sharded stack wires them: the o projection reads, for each
    rank r, the first o-slice-width columns of r's qkv rows; down reads the
    gate output."""
    from popcorn_b200.tp import shard_bounds

    h = x
    for w in full_layers:
        a = pc.dequantize_matmul(h, *w["qkv"])
        cols = []
        for r in range(world):
            qlo, _ = shard_bounds(dims["qkv"], world, r)
            olo, ohi = shard_bounds(dims["hidden"], world, r)
            cols.append(a[:, qlo:qlo + (ohi - olo)])
        h1 = pc.dequantize_matmul(torch.cat(cols, dim=1).contiguous(), *w["o"])
        g = pc.dequantize_matmul(h1, *w["gate"])
        pc.dequantize_matmul(h1, *w["up"])
        h = pc.dequantize_matmul(g, *w["down"])
    return h


def time_stack(torch, pc, M, layers, rank, world, device, peaks, dist_on):
    """One pass of the 32-layer stack = one step; K passes from one CUDA graph."""
    from popcorn_b200.tp import STACK_7B, LinearStack, PeerGroup

    check_layers = 2 if world > 1 else 0
    shards, full_layers = stack_shards(torch, pc, STACK_7B, layers, rank, world, device, 4242, check_layers)
    peer = PeerGroup(M, STACK_7B["hidden"], device) if (world > 1 and M <= 4) else None
    stack = LinearStack(shards, M, STACK_7B, device, peer=peer)
    gx = torch.Generator(device=device)
    gx.manual_seed(77 + M)
    x = torch.randn((M, STACK_7B["hidden"]), generator=gx, device=device)
    stream = torch.cuda.Stream()
    passes = 8
    with torch.cuda.stream(stream):
        for _ in range(3):
            stack(x)
    stream.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for _ in range(passes):
            stack(x)
    with torch.cuda.stream(stream):
        graph.replay()
    stream.synchronize()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    if dist_on:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        lead_in(torch)
        start.record(stream)
        graph.replay()
        end.record(stream)
    torch.cuda.synchronize()
    ms = max_over_ranks(torch, start.elapsed_time(end), dist_on, device) / passes
    errs = pc.device_errors()
    del graph
    parity = None
    if check_layers:
        # The first layers of the sharded stack (same shards, same collectives)
        # against the same layers unsharded on this GPU.
        head = LinearStack(shards[:check_layers], M, STACK_7B, device, peer=peer)
        with torch.cuda.stream(stream):
            got = head(x).clone()
            ref = stack_reference(torch, pc, full_layers, x, world, STACK_7B)
        torch.cuda.synchronize()
        err = float((got.double() - ref.double()).abs().max() / ref.double().abs().max())
        tol = 1e-5 if M <= 4 else 2e-3
        parity = {"what": f"first {check_layers} layers vs the same layers unsharded on one GPU",
                  "max_err": err, "tol": tol, "ok": bool(err <= tol) and pc.device_errors() == 0}
        del head, full_layers
    wbytes = stack.weight_bytes()
    if dist_on:
        t = torch.tensor([wbytes], dtype=torch.int64, device=device)
        torch.distributed.all_reduce(t)
        wbytes = int(t.item())
    gbs = wbytes / (ms * 1e-3) / 1e9
    res = {"value": round(gbs, 2), "unit": "GB/s", "M": M, "layers": layers, "ms_per_pass": round(ms, 4),
           "weight_bytes_per_pass": wbytes, "passes_timed": passes,
           "roofline": {"bound": "hbm", "achieved": round(gbs, 2), "peak": round(peaks["hbm"] * world, 1),
                        "unit": "GB/s", "frac": round(gbs / (peaks["hbm"] * world), 4),
                        "peak_source": peaks["source"] + (f" x{world}" if world > 1 else "")},
           "launches_per_pass": stack.launches_per_pass(),
           "row_parallel_sum": ("single GPU" if world == 1 else
                                "fused into the GEMV (tagged NVLink peer stores)" if stack.peer is not None
                                else "NCCL all-reduce"),
           "device_error_bits": errs}
    if parity is not None:
        res["tp_parity"] = parity
    if M > 1:
        res["tflops"] = round(2.0 * M * wbytes / (ms * 1e-3) / 1e12, 2)
    del stack, shards, peer
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    return res


def run_ours(args):
    import torch

    import popcorn_b200 as pc

    rank, world, local = dist_env()
    dist_on = world > 1
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if dist_on:
        import datetime

        torch.distributed.init_process_group("nccl", device_id=device, timeout=datetime.timedelta(seconds=120))
    peaks = measured_peaks()
    l2 = torch.cuda.get_device_properties(device).L2_cache_size
    pool = 2.5 * l2

    wl = WORKLOADS[args.workload]
    if wl.get("op") or wl.get("mlp"):
        # The weight-side kernels and the fused MLP front are single-GPU workloads.
        if world > 1:
            raise SystemExit(f"--workload {args.workload} runs on one GPU")
        setup = (OpSetup if wl.get("op") else MlpSetup)(torch, pc, wl, device, pool)
    else:
        setup = Setup(torch, pc, wl, rank, world, device, pool)
    sampler = ClockSampler(device)
    sampler.start()
    ms, clocks = time_graph(torch, setup, args.steps, args.warmup, args.soak_s, sampler, dist_on)
    sampler.stop()
    ms = max_over_ranks(torch, ms, dist_on, device)
    ms_step = ms / args.steps
    value = throughput(wl, ms_step)
    launches = setup.launches_per_step()
    tp_parity = None
    if dist_on:
        stream = torch.cuda.Stream()
        with torch.cuda.stream(stream):
            tp_parity = setup.tp_parity(stream.cuda_stream)
        flag = torch.tensor([0 if tp_parity["ok"] else 1], dtype=torch.int32, device=device)
        torch.distributed.all_reduce(flag)
        tp_parity["ranks_failing"] = int(flag.item())
        tp_parity["ok"] = tp_parity["ok"] and tp_parity["ranks_failing"] == 0

    line = {
        "metric": METRIC,
        "value": round(value, 2),
        "unit": wl["unit"],
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms_step, 6),
        "higher_is_better": True,
        "scaling": "strong" if world > 1 else "weak",
        "vs_baseline": None,
        "dtype": compute_dtype(setup.path(), wl["M"], wl["K"], bool(wl.get("group_size"))),
        "data": "synthetic: X ~ N(0,1), W ~ N(0,0.02) (torch.randn, fixed seed), int8 per-row via popcornQuantize_f32i8",
        "config": {
            "workload": f"{args.workload} M={wl['M']} K={wl['K']} N={wl['N']}",
            "M": wl["M"], "K": wl["K"], "N": wl["N"],
            "parallelism": (f"column-parallel N-shard x{world} + " +
                            ("all-gather fused into the GEMV (tagged NVLink peer stores)" if setup.fused is not None
                             else "NCCL all-gather")) if world > 1 else "single GPU",
            "path": setup.path(),
            "l2": f"weights rotate over {setup.sets} sets "
                  f"({setup.sets * setup.Nl * wl['K'] / 1e6:.0f} MB per rank > 2x L2 {l2 / 1e6:.0f} MB)",
            "timing": "K steps replayed from one CUDA graph; CUDA events on the launching stream bracket exactly "
                      "those K steps (a ~1 ms spin kernel ahead of the start event keeps host submission latency "
                      "out); max over ranks",
        },
        "gpu_launches": launches * args.steps,
        "roofline": roofline(dict(wl, N=setup.Nl), ms_step, peaks, args.workload) if world == 1 else
        roofline(wl, ms_step, dict(peaks, hbm=peaks["hbm"] * world, tc=peaks["tc"] * world), args.workload),
        "clocks": clocks,
    }
    if tp_parity is not None:
        line["tp_parity"] = tp_parity

    if not args.no_e2e:
        e2e_steps = min(args.steps, 2000)
        ems, h2d, d2h = time_e2e(torch, setup, e2e_steps, max(3, args.warmup), dist_on)
        ems = max_over_ranks(torch, ems, dist_on, device)
        line["e2e"] = {"value": round(throughput(wl, ems / e2e_steps), 2), "unit": wl["unit"],
                       "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "steps": e2e_steps,
                       "ms_per_step": round(ems / e2e_steps, 6),
                       "how": "pinned H2D of x (cudaMemcpyAsync) + " + (
                           "popcornDequantizeMatmulAllGather_i8f32" if setup.fused is not None else
                           "popcornDequantizeMatmul_i8f32" + (" + NCCL all-gather" if world > 1 else ""))
                              + " via ctypes + pinned D2H of the full y, stream-synchronized every step"}

    if world == 1 and rank == 0:
        extras = {}
        for name in [e for e in args.extras.split(",") if e in WORKLOADS and e != args.workload]:
            ewl = WORKLOADS[name]
            if ewl.get("mlp"):
                es = MlpSetup(torch, pc, ewl, device, pool)
            elif ewl.get("op"):
                es = OpSetup(torch, pc, ewl, device, pool)
            else:
                es = Setup(torch, pc, ewl, 0, 1, device, pool)
            esteps = 200 if ewl["bound"] == "hbm" else 20
            ems, _ = time_graph(torch, es, esteps, 3, 0.0, None, False)
            eval_ = throughput(ewl, ems / esteps)
            extras[name] = {"value": round(eval_, 2), "unit": ewl["unit"], "M": ewl["M"], "K": ewl["K"],
                            "N": ewl["N"], "path": es.path(), "steps": esteps,
                            "ms_per_step": round(ems / esteps, 6),
                            "roofline": roofline(ewl, ems / esteps, peaks, name)}
            del es
            if ewl.get("mlp"):
                eu = MlpSetup(torch, pc, ewl, device, pool, fused=False)
                ums, _ = time_graph(torch, eu, esteps, 3, 0.0, None, False)
                extras[name]["unfused_ms_per_step"] = round(ums / esteps, 6)
                extras[name]["unfused"] = "torch RMSNorm + 2 x popcornDequantizeMatmul_i8f32 + torch silu * up"
                del eu
            torch.cuda.empty_cache()
        if extras:
            line["extra_workloads"] = extras
        if not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(torch, setup, wl)

    if args.stack != "none":
        stack = {}
        for m in [int(v) for v in args.stack.split(",") if v]:
            stack[f"m{m}"] = time_stack(torch, pc, m, args.stack_layers, rank, world, device, peaks, dist_on)
        line["stack_7b_linear"] = dict(
            stack, config="32 layers x (qkv 4096->12288, o 4096->4096, gate and up 4096->11008, down 11008->4096), "
                          "column-parallel qkv/gate/up, row-parallel o/down, one pass per step from a CUDA graph, "
                          "max over ranks" if args.stack_layers == 32 else f"{args.stack_layers} layers")

    if rank == 0:
        print(json.dumps(line), flush=True)
    if dist_on:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


# ---------------------------------------------------------------------------
# Reference arm: popcorn's own CPU loop on the host cores (rank 0 only).
# ---------------------------------------------------------------------------
def run_reference(args):
    rank, world, local = dist_env()
    if rank != 0:
        return
    import numpy as np

    import oracle

    wl = WORKLOADS[args.workload]
    M, K, N = wl["M"], wl["K"], wl["N"]
    threads = host_threads()
    use_ref = oracle.have_ref_loops()
    kind = "reference" if use_ref else "port"
    x = oracle.fill_normal(M * K, 0, 1.0).reshape(M, K)
    w = oracle.fill_normal(N * K, 1, 0.02).reshape(N, K)
    q, s = oracle.quantize(w)

    def call(rows):
        if use_ref:
            oracle.ref_dequant_matmul(x, q[:rows], s[:rows], threads=threads)
        else:
            oracle.dequant_matmul(x, q[:rows], s[:rows], threads=threads)

    t0 = time.perf_counter()
    call(N)
    full = time.perf_counter() - t0
    # Bound the run: each step is the full call if K steps fit in ~90 s,
    # otherwise a leading block of output channels (same per-row work).
    budget = 90.0 / max(1, args.steps + args.warmup)
    rows = N if full <= budget else max(threads, int(N * budget / full))
    for _ in range(args.warmup):
        call(rows)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        call(rows)
    dt = (time.perf_counter() - t0) / args.steps
    if wl["unit"] == "GB/s":
        value = rows * K / dt / 1e9
    else:
        value = 2.0 * M * rows * K / dt / 1e12
    sample = (f"each step: popcorn test loop on M={M} K={K} N={rows} of {N} rows, "
              f"{dt * 1e3:.3f} ms, {threads} threads, wall clock")
    line = {
        "metric": METRIC, "impl": "reference", "value": round(value, 4), "unit": wl["unit"], "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt * 1e3 * N / rows, 6),
        "higher_is_better": True, "scaling": "strong" if world > 1 else "weak", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic: X ~ N(0,1), W ~ N(0,0.02) (SplitMix64 + Irwin-Hall), int8 per-row",
        "config": {"workload": f"{args.workload} M={M} K={K} N={N}", "M": M, "K": K, "N": N,
                   "parallelism": "host cores of rank 0"},
        "cpu_baseline": {"value": round(value, 4), "unit": wl["unit"], "cores": threads, "kind": kind,
                         "sample": sample},
        "e2e": {"value": round(value, 4), "unit": wl["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "gpu_launches": 0,
    }
    try:
        line["reference_gpu_kernel"] = reference_gpu_kernel(args, wl, x, q, s)
    except Exception as e:  # noqa: BLE001 - the CPU arm stands on its own
        line["reference_gpu_kernel"] = {"unavailable": str(e)[:200]}
    print(json.dumps(line), flush=True)


def reference_gpu_kernel(args, wl, x, q, s):
    """popcorn's own CUDA kernel (src/quantize.cu rebuilt for sm_100a), timed
    like ours: weights rotated beyond L2, K launches from one CUDA graph."""
    import torch

    import oracle

    if not oracle.have_popcorn_ref_gpu() or not torch.cuda.is_available():
        return {"unavailable": "oracle/_ref/libpopcorn_ref.so or GPU missing"}
    lib = oracle.popcorn_ref_gpu()
    dev = torch.device("cuda", 0)
    M, K, N = wl["M"], wl["K"], wl["N"]
    l2 = torch.cuda.get_device_properties(dev).L2_cache_size
    sets = max(2, math.ceil(2.5 * l2 / (N * K)))
    qd = torch.from_numpy(q).to(dev)
    sd = torch.from_numpy(s).to(dev)
    qs = [qd] + [qd.clone() for _ in range(sets - 1)]
    xd = torch.from_numpy(x).to(dev)
    out = torch.empty((M, N), dtype=torch.float32, device=dev)
    steps = min(args.steps, 200)
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        for i in range(3):
            assert lib.popcornDequantizeMatmul_i8f32(out.data_ptr(), xd.data_ptr(), qs[i % sets].data_ptr(),
                                                     sd.data_ptr(), M, N, K, stream.cuda_stream) == 0
    stream.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        for i in range(steps):
            lib.popcornDequantizeMatmul_i8f32(out.data_ptr(), xd.data_ptr(), qs[i % sets].data_ptr(),
                                              sd.data_ptr(), M, N, K, stream.cuda_stream)
    with torch.cuda.stream(stream):
        g.replay()
    stream.synchronize()
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        a.record(stream)
        g.replay()
        b.record(stream)
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / steps
    ref = oracle.dequant_matmul(x, q, s, fused=True, threads=host_threads())
    got = out.cpu().numpy()
    return {"value": round(throughput(wl, ms), 2), "unit": wl["unit"], "ms_per_step": round(ms, 6),
            "steps": steps, "what": "popcorn src/quantize.cu dequantizeMatmulKernel_i8f32, nvcc -O3 sm_100a",
            "normwise_err_vs_oracle": oracle.normwise_rel_err(got, ref)}


def main():
    args = parse_args()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
