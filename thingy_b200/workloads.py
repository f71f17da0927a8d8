"""Seeded synthetic inputs for the five workloads of this path.

There is no public dataset for this op; every input is synthetic with the
shapes and value distributions below. Generation uses a seeded
torch.Generator on the requested device, so a CPU generation is reproducible
bit for bit (parity tests build inputs on the CPU and copy them to the GPU).

  token_4096x4096        per-token FP8, x ~ N(0,1) [4096, 4096], eps 1e-6
  g128_16384x7168        1x128 FP8 (DeepSeek-V3 shape), x ~ N(0,1) with
                         round(0.001*H) outlier channels x50, column-major
                         fp32 scales [H/128, M], eps 1e-6
  residual_token_32768x8192
                         residual add + per-token FP8, x ~ N(0,1),
                         residual ~ N(0, 4) (sigma 2), eps 1e-5, residual_out
  rmsnorm_bf16_16384x7168
                         the standalone bf16 RMSNorm (rms_norm_reference,
                         bf16 out), x ~ N(0,1), config 2's shape
  rmsnorm_f32_MxH        the standalone fp32 RMSNorm of the reference's older
                         baseline (x, w ~ N(0,1) fp32, eps 1e-5) at the shapes
                         of its published sweep, M in {1024, 4096, 16384},
                         H in {1024, 3072, 7168}
  mx32_decode_5120       decode-size MXFP8: M in {1, 8, 32, 128}, H 5120,
                         x ~ Student-t(nu=4), e8m0 scales per 32 elements in
                         the Blackwell swizzled layout, eps 1e-6
  g128_sharded_262144x8192
                         1x128 FP8 over row shards, x ~ N(0,1) with
                         round(0.001*H) outlier channels x50, column-major
                         fp32 scales, eps 1e-6
  prologue_mx32_5120x5120
                         config 4's decode MXFP8 rows (M in {1, 8, 32, 128},
                         H = K = 5120, Student-t) fed to a 5120 x 5120
                         block-scaled FP8 GEMM: RMSNorm -> MXFP8 -> GEMM in
                         one kernel; the GEMM weight is bf16 0.05*N(0,1)
                         quantized to MXFP8 by this path
Weights are bf16 1 + 0.1*N(0,1) everywhere.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class Workload:
    name: str
    M: int
    H: int
    eps: float
    group_size: int | None  # None = one scale per row
    scale_format: str
    scale_layout: str
    residual: bool
    dist: str  # "normal", "outliers", "student_t"
    kind: str = "fused"  # "fused" (bf16 -> fp8), "rms_f32" / "rms_bf16" (standalone RMSNorm),
    #                      "bwd" (backward: gradients of the fused path) or "prologue"
    #                      (RMSNorm -> MXFP8 -> GEMM with an N x H weight, one kernel)
    N: int = 0           # GEMM output columns ("prologue" only)

    def bytes_moved(self, M: int | None = None) -> int:
        """Algorithmic HBM bytes of one pass: inputs read once, outputs written once.

        x (+ residual) bf16 read, weight read once, q e4m3 written, scales
        written (4 B fp32 or 1 B e8m0 per group), residual_out bf16 written
        when there is a residual. Follows fused_memory_bytes
        (src/cutie/rms_norm/bench.py:149-158) minus the normalized output,
        which these workloads do not request.
        """
        M = self.M if M is None else M
        H = self.H
        if self.kind == "prologue":
            # read x, the norm weight, the e4m3 GEMM weight and its e8m0
            # scales; write D (bf16). The FP8 activation stays on chip.
            return 2 * M * H + 2 * H + self.N * H + self.N * (H // 32) + 2 * M * self.N
        if self.kind == "rms_f32":  # utils.py:10-19: x and out fp32, weight once
            return 2 * M * H * 4 + H * 4
        if self.kind == "rms_bf16":  # x and out bf16, weight once
            return 2 * M * H * 2 + H * 2
        if self.kind == "bwd":
            # read d_normalized, r [, d_residual_out], weight; write dx, d_weight
            # [, FP8 codes + scales of dx]. The per-CTA partial sums of d_weight
            # in the workspace are not counted (not an input or output).
            total = 2 * M * H + 2 * M * H + 2 * H + 2 * M * H + 2 * H
            if self.residual:
                total += 2 * M * H
            if self.group_size:
                total += M * H + (1 if self.scale_format == "e8m0" else 4) * M * -(-H // 128)
            return total
        groups = 1 if not self.group_size else -(-H // self.group_size)
        scale_bytes = 1 if self.scale_format == "e8m0" else 4
        total = 2 * M * H + 2 * H + M * H + scale_bytes * M * groups
        if self.residual:
            total += 2 * M * H + 2 * M * H
        return total


WORKLOADS = {
    w.name: w
    for w in (
        Workload("token_4096x4096", 4096, 4096, 1e-6, None, "fp32", "row", False, "normal"),
        Workload("g128_16384x7168", 16384, 7168, 1e-6, 128, "fp32", "col", False, "outliers"),
        Workload("residual_token_32768x8192", 32768, 8192, 1e-5, None, "fp32", "row", True,
                 "normal"),
        Workload("mx32_decode_5120", 128, 5120, 1e-6, 32, "e8m0", "mx", False, "student_t"),
        Workload("g128_sharded_262144x8192", 262144, 8192, 1e-6, 128, "fp32", "col", False,
                 "outliers"),
        Workload("bwd_residual_g128_16384x7168", 16384, 7168, 1e-6, 128, "fp32", "col", True,
                 "normal", kind="bwd"),
        Workload("prologue_mx32_5120x5120", 128, 5120, 1e-6, 32, "e8m0", "mx", False,
                 "student_t", kind="prologue", N=5120),
        *(
            Workload(f"rmsnorm_f32_{m}x{h}", m, h, 1e-5, None, "fp32", "row", False, "normal",
                     kind="rms_f32")
            for m in (1024, 4096, 16384)
            for h in (1024, 3072, 7168)
        ),
        Workload("rmsnorm_bf16_16384x7168", 16384, 7168, 1e-6, None, "fp32", "row", False,
                 "normal", kind="rms_bf16"),
    )
}

DECODE_ROWS = (1, 8, 32, 128)


def _weight(H: int, gen: torch.Generator, device) -> torch.Tensor:
    return (1.0 + 0.1 * torch.randn(H, generator=gen, device=device)).to(torch.bfloat16)


def _student_t(shape, nu: int, gen: torch.Generator, device) -> torch.Tensor:
    # t = Z / sqrt(chi2_nu / nu), chi2_nu = sum of nu squared standard normals
    z = torch.randn(shape, generator=gen, device=device)
    chi2 = torch.zeros(shape, device=device)
    for _ in range(nu):
        chi2 += torch.randn(shape, generator=gen, device=device).square()
    return z / torch.sqrt(chi2 / nu)


def make_inputs(w: Workload, M: int | None = None, *, device="cpu", seed: int = 0,
                row_offset: int = 0) -> dict:
    """x (+ residual) [M, H] bf16 and weight [H] bf16 for workload ``w``.

    The outlier channels and the weight depend only on (seed, H), so row
    shards generated with different ``row_offset`` share them. ``row_offset``
    reseeds the row data per shard (shard inputs are independent draws).
    """
    M = w.M if M is None else M
    H = w.H
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    if w.kind == "bwd":  # r (= residual_out of the forward), gradients ~N(0,1)
        weight = _weight(H, gen, device)
        if row_offset:
            gen.manual_seed(seed * 1_000_003 + row_offset)
        r = (torch.randn((M, H), generator=gen, device=device)
             + 2.0 * torch.randn((M, H), generator=gen, device=device)).to(torch.bfloat16)
        out = {"r": r, "weight": weight, "eps": w.eps,
               "d_normalized": torch.randn((M, H), generator=gen, device=device).to(torch.bfloat16)}
        if w.residual:
            out["d_residual_out"] = torch.randn((M, H), generator=gen, device=device).to(
                torch.bfloat16)
        return out
    if w.kind == "rms_bf16":  # rms_norm_reference (bench.py:58-65) on bf16 rows
        weight = _weight(H, gen, device)
        if row_offset:
            gen.manual_seed(seed * 1_000_003 + row_offset)
        x = torch.randn((M, H), generator=gen, device=device).to(torch.bfloat16)
        return {"x": x, "weight": weight, "eps": w.eps}
    if w.kind == "rms_f32":  # utils.py:38-59: randn x and weight, fp32
        if row_offset:
            gen.manual_seed(seed * 1_000_003 + row_offset)
        x = torch.randn((M, H), generator=gen, device=device)
        return {"x": x, "weight": torch.randn(H, generator=gen, device=device), "eps": w.eps}
    if w.kind == "prologue":  # the decode rows plus the GEMM weight
        weight = _weight(H, gen, device)
        gemm_w = (0.05 * torch.randn((w.N, H), generator=gen, device=device)).to(torch.bfloat16)
        if row_offset:
            gen.manual_seed(seed * 1_000_003 + row_offset)
        x = _student_t((M, H), 4, gen, device)
        return {"x": x.to(torch.bfloat16), "weight": weight, "eps": w.eps, "gemm_weight": gemm_w}
    weight = _weight(H, gen, device)
    outliers = None
    if w.dist == "outliers":
        k = max(1, round(0.001 * H))
        outliers = torch.randperm(H, generator=gen, device=device)[:k]
    if row_offset:
        gen.manual_seed(seed * 1_000_003 + row_offset)
    if w.dist == "student_t":
        x = _student_t((M, H), 4, gen, device)
    else:
        x = torch.randn((M, H), generator=gen, device=device)
    if outliers is not None:
        x[:, outliers] *= 50.0
    out = {"x": x.to(torch.bfloat16), "weight": weight, "eps": w.eps}
    if w.residual:
        out["residual"] = (2.0 * torch.randn((M, H), generator=gen, device=device)).to(
            torch.bfloat16
        )
    return out
