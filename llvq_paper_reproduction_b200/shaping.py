"""Wrappers around the Λ24 quantizer: spherical shaping with a global scale
(the reference's Gaussian evaluation) and shape-gain quantization with a
scalar gain code matched to the chi distribution with 24 degrees of freedom.

Spherical shaping follows the reference notebook
notebooks/recreate_figure1_gaussian_sqnr.ipynb (cells 5 and 7):
``ideal_gaussian_source_scale`` picks beta = sqrt(24 sigma^2 / E||y/sqrt 8||^2)
over the finite ball codebook, blocks are quantized as Q(w / beta) and
reconstructed as beta * dequantize(index); quality is reported as
SQNR_bits = -1/2 log2(MSE) (impl/gaussian_baseline_quantizers.py:28-29).

Shape-gain has no reference implementation (the reference README lists it
but the package does not exist); it is defined here as:
  * shape: the nearest point of one shell m (the reference search restricted
    to shells m..m, i.e. the largest correlation <x, y>), direction
    u = y / |y|; or, multi-shell, the point of shells m_lo..m_hi with the
    largest correlation per unit norm <x, y> / |y| (fp64, ties in the
    reference's loop order; generated "angular" search code);
  * gain: g = <x, u> (the least-squares gain for that direction), coded with
    a b-bit Lloyd-Max quantizer designed for the chi(24) density scaled by
    sigma (the norm of a 24-D N(0, sigma^2 I) block);
  * index = shape_index * 2^b + gain_index, reconstruction g_q * u;
  * optional post-shape gain code (fit_gain_code): the levels refitted as the
    mean projection <x, u> of each gain cell on a sample, given the shapes
    the quantizer picked -- the MSE-optimal scale of every cell's blocks.
The shape search and the gain code run in one library call
(llvq_quantize_gain): the finalize kernel that ranks the winning codeword
also forms g = <x, y> / |y| in fp64 (the compensated projection of the
reference score) and codes it against fp64 thresholds.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from functools import lru_cache

import numpy as np
import torch

from .quantizer import LeechLatticeVectorQuantizerGpu
from .tables import DIM, leech_shell_counts


def mse_to_sqnr_bits(mse: float) -> float:
    """SQNR in bits, -1/2 log2(MSE) (reference: impl/gaussian_baseline_quantizers.py:28-29)."""
    return -0.5 * math.log2(mse)


def mse_to_sqnr_db(mse: float) -> float:
    return 10.0 * math.log10(1.0 / mse)


def ideal_gaussian_source_scale(q: LeechLatticeVectorQuantizerGpu, variance: float = 1.0) -> float:
    """beta matching the ball codebook's mean squared norm (shell m has squared
    norm 2m after the 1/sqrt(8) scale) to a 24-D Gaussian source of the given
    variance."""
    weighted = sum(2.0 * shell * count for shell, count in q.shell_counts.items())
    return math.sqrt(DIM * variance / (weighted / q.total_count))


class SphericalShaping:
    """Global-beta quantizer over the ball codebook shells min..max."""

    def __init__(self, quantizer: LeechLatticeVectorQuantizerGpu, variance: float = 1.0):
        self.q = quantizer
        self.beta = ideal_gaussian_source_scale(quantizer, variance)

    def quantize(self, w: torch.Tensor) -> torch.Tensor:
        # true fp32 division by fp32(beta), as numpy evaluates w / beta for a
        # float32 array (torch's scalar division would multiply by a rounded
        # reciprocal instead)
        w = w.to(device=self.q.device, dtype=torch.float32)
        return self.q.quantize(w / torch.tensor(self.beta, dtype=torch.float32, device=w.device))

    def dequantize(self, indices: torch.Tensor) -> torch.Tensor:
        return self.beta * self.q.dequantize(indices)

    def evaluate(self, w: torch.Tensor) -> dict:
        """MSE per dimension and SQNR of w [n, 24] (the notebook's evaluate_spherical_shaping):
        reconstruction in float64 from the CPU-API dequantized values."""
        w = w.to(device=self.q.device, dtype=torch.float32)
        idx = self.quantize(w)
        lat = self.q.dequantize_lattice(idx).to(torch.float64)
        recon = self.beta * (lat * (1.0 / math.sqrt(8.0)))
        err = (w.to(torch.float64) - recon).pow(2).sum().item()
        mse = err / (w.shape[0] * DIM)
        return {"indices": idx, "mse": mse, "sqnr_bits": mse_to_sqnr_bits(mse), "sqnr_db": mse_to_sqnr_db(mse),
                "beta": self.beta, "shape_bits": self.q.shape_bits}


# ------------------------------------------------------------------ gain code

@lru_cache(maxsize=64)
def chi_lloyd_max(bits: int, dof: int = DIM, iters: int = 400) -> tuple[np.ndarray, np.ndarray]:
    """Lloyd-Max reconstruction levels and decision thresholds (ascending)
    for the chi distribution with `dof` degrees of freedom (unit sigma).

    The density is evaluated on a fine grid; each iteration places the
    thresholds at the midpoints of the levels and moves every level to the
    conditional mean of its cell."""
    n = 1 << bits
    grid = np.linspace(1e-6, math.sqrt(dof) + 12.0, 200_001)
    logpdf = (dof - 1) * np.log(grid) - grid * grid / 2.0
    pdf = np.exp(logpdf - logpdf.max())
    cdf = np.cumsum(pdf)
    first = np.cumsum(pdf * grid)
    total = cdf[-1]
    # start from equal-probability cells
    edges = np.interp(np.linspace(0, total, n + 1), cdf, grid)
    levels = 0.5 * (edges[:-1] + edges[1:])
    for _ in range(iters):
        thr = 0.5 * (levels[:-1] + levels[1:])
        idx = np.searchsorted(grid, thr)
        bounds = np.concatenate([[0], idx, [grid.size]])
        new = np.empty_like(levels)
        for i in range(n):
            lo, hi = bounds[i], bounds[i + 1]
            mass = cdf[hi - 1] - (cdf[lo - 1] if lo else 0.0)
            mom = first[hi - 1] - (first[lo - 1] if lo else 0.0)
            new[i] = mom / mass if mass > 0 else levels[i]
        if np.max(np.abs(new - levels)) < 1e-12:
            levels = new
            break
        levels = new
    return levels, 0.5 * (levels[:-1] + levels[1:])


def lloyd_max_empirical(sample: np.ndarray, levels0: np.ndarray, iters: int = 500,
                        tol: float = 1e-13) -> tuple[np.ndarray, np.ndarray]:
    """Lloyd-Max levels and thresholds (ascending) for the empirical
    distribution of a 1-D sample, started from levels0.

    Cells follow the gain coder's rule: code i holds the values in
    (thr[i-1], thr[i]] (the number of thresholds strictly below the value).
    Each iteration places the thresholds at the midpoints of the levels and
    moves every level with a non-empty cell to the mean of the sample values
    in it, with sorted data and prefix sums (O(levels log n) per iteration).
    The result is the last iteration's pair: thresholds at the midpoints of
    the previous levels and levels at the means of the cells they bound, so
    every non-empty cell's level is exactly its mean even when the iteration
    stops before it converges."""
    s = np.sort(np.asarray(sample, dtype=np.float64).ravel())
    if s.size == 0:
        raise ValueError("empty sample")
    prefix = np.concatenate([[0.0], np.cumsum(s)])
    levels = np.sort(np.asarray(levels0, dtype=np.float64))
    thr = 0.5 * (levels[:-1] + levels[1:])
    for _ in range(max(1, iters)):
        thr = 0.5 * (levels[:-1] + levels[1:])
        bounds = np.concatenate([[0], np.searchsorted(s, thr, side="right"), [s.size]])
        count = np.diff(bounds)
        mean = (prefix[bounds[1:]] - prefix[bounds[:-1]]) / np.maximum(count, 1)
        new = np.where(count > 0, mean, levels)
        new = np.maximum.accumulate(new)  # an empty cell keeps its level; stay ordered
        done = np.max(np.abs(new - levels)) <= tol * max(1.0, float(np.max(np.abs(levels))))
        levels = new
        if done:
            break
    return levels, thr


@dataclass(frozen=True)
class RateSplit:
    shell: int
    shape_bits: int
    gain_bits: int

    @property
    def bits_per_dim(self) -> float:
        return (self.shape_bits + self.gain_bits) / DIM


def rate_split(bits_per_dim: float, min_gain_bits: int = 3, max_shape_bits: int = 62) -> RateSplit:
    """Largest single shell whose index fits the budget with at least
    `min_gain_bits` left for the gain; the remaining bits go to the gain."""
    budget = int(round(bits_per_dim * DIM))
    counts = leech_shell_counts(60)
    best = None
    for m in range(2, 61):
        sb = math.ceil(math.log2(counts[m]))
        if sb > max_shape_bits or sb + min_gain_bits > budget:
            break
        best = RateSplit(m, sb, budget - sb)
    if best is None:
        raise ValueError(f"no shell fits {bits_per_dim} bits/dim")
    return best


# Multi-shell shape codebooks with generated angular search code, by rate:
# (min shell, max shell, gain bits); shells 2..5 have 2^32.2 points (33 shape
# bits), 2..10 have 2^43.6 (44 shape bits).
MULTI_SHELL_SPLITS = {1.5: (2, 5, 3), 2.0: (2, 10, 4)}


class ShapeGainQuantizer:
    """Shape from one shell (min_shell = shell, the default) or from shells
    min_shell..shell by correlation per unit norm, with a chi-matched scalar
    gain (no reference counterpart; see the module docstring)."""

    def __init__(self, shell: int, gain_bits: int, sigma: float = 1.0, device="cuda", use_cache: bool = False,
                 min_shell: int | None = None):
        lo = shell if min_shell is None else min_shell
        self.shape = LeechLatticeVectorQuantizerGpu(max_shell=shell, min_shell=lo, device=device,
                                                    use_cache=use_cache)
        self.shell = shell
        self.min_shell = lo
        self.multi_shell = lo < shell
        self.gain_bits = gain_bits
        self.sigma = sigma
        levels, thr = chi_lloyd_max(gain_bits)
        self.levels = torch.tensor(levels * sigma, dtype=torch.float32, device=self.shape.device)
        self.thresholds = torch.tensor(thr * sigma, dtype=torch.float64, device=self.shape.device)
        self.norm = math.sqrt(2.0 * shell)  # |y| / sqrt(8) for every point of the shell

    @classmethod
    def for_rate(cls, bits_per_dim: float, sigma: float = 1.0, device="cuda",
                 multi_shell: bool = False) -> "ShapeGainQuantizer":
        if multi_shell:
            if bits_per_dim not in MULTI_SHELL_SPLITS:
                raise ValueError(f"no multi-shell split for {bits_per_dim} bits/dim "
                                 f"(have {sorted(MULTI_SHELL_SPLITS)})")
            lo, hi, gb = MULTI_SHELL_SPLITS[bits_per_dim]
            return cls(hi, gb, sigma, device, min_shell=lo)
        split = rate_split(bits_per_dim)
        return cls(split.shell, split.gain_bits, sigma, device)

    @classmethod
    def for_rate_post_shape(cls, bits_per_dim: float, sigma: float = 1.0, device="cuda", multi_shell: bool = False,
                            design_blocks: int = 65536, design_seed: int = 7) -> "ShapeGainQuantizer":
        """for_rate with the gain code fitted after the shape quantizer
        (fit_gain_code) on design_blocks N(0, sigma^2) blocks from a seeded
        generator."""
        sg = cls.for_rate(bits_per_dim, sigma, device, multi_shell)
        g = torch.Generator().manual_seed(design_seed)
        sg.fit_gain_code(torch.randn((design_blocks, DIM), generator=g, dtype=torch.float32) * sigma)
        return sg

    def projections(self, x: torch.Tensor, shape_idx: torch.Tensor,
                    row_sigma: torch.Tensor | None = None) -> torch.Tensor:
        """<x, y> / |y| (fp64) of every block with its shape codeword y,
        divided by row_sigma when given: the value the gain code codes."""
        dev = self.shape.device
        x = torch.as_tensor(x, device=dev).reshape(-1, DIM).to(torch.float64)
        y = self.shape.dequantize_lattice(shape_idx.reshape(-1).to(dev)).to(torch.float64)
        c = (x * y).sum(dim=-1) / y.pow(2).sum(dim=-1).sqrt()
        if row_sigma is not None:
            sig = torch.broadcast_to(torch.as_tensor(row_sigma, dtype=torch.float32, device=dev),
                                     shape_idx.shape).reshape(-1).to(torch.float64)
            c = c / sig
        return c

    def fit_gain_code(self, x: torch.Tensor, row_sigma: torch.Tensor | None = None, iters: int = 500) -> dict:
        """Optimal post-shape gain scales: refit the gain code to the
        projections c = <x, u> of sample blocks on the directions u that the
        shape quantizer picks for them.

        Given the shapes, the reconstruction of a block with gain code i is
        l_i u, and sum |x - l_i u|^2 = sum |x|^2 - 2 l_i c + l_i^2 over the
        blocks of cell i is smallest at l_i = mean(c | cell i); the best
        thresholds for given levels are their midpoints.  The code designed
        for chi(24) (the norm |x|) ignores that c = |x| cos(theta) is smaller
        than |x| by the shape's angular error; a Lloyd-Max iteration on the
        sample of c, started from the chi(24) levels, fixes both conditions.
        The shape search does not depend on the gain code (below), so one
        pass of the shape quantizer over the sample suffices.

        Joint (shape, gain) choice: with positive levels, min over (u, l) of
        |x|^2 - 2 l <x, u> + l^2 takes, for every l, the u with the largest
        <x, u>, so the sequential choice (largest correlation per unit norm,
        then the nearest level to c) is the joint optimum (Sabin and Gray,
        IEEE Trans. ASSP 32(3), 1984)."""
        sidx, _ = self.quantize_parts(x, row_sigma)
        ok = sidx.reshape(-1) >= 0
        c = self.projections(x, sidx, row_sigma)[ok].cpu().numpy()
        start = self.levels.double().cpu().numpy()
        levels, thr = lloyd_max_empirical(c, start, iters=iters)
        if np.any(levels <= 0):
            raise ValueError("the fitted gain code has a non-positive level")
        self.levels = torch.tensor(levels, dtype=torch.float32, device=self.shape.device)
        self.thresholds = torch.tensor(thr, dtype=torch.float64, device=self.shape.device)
        return {"blocks": int(c.size), "levels": levels, "thresholds": thr,
                "mean_projection": float(c.mean()), "chi_levels": start}

    @property
    def bits(self) -> int:
        return self.shape.shape_bits + self.gain_bits

    def quantize_parts(self, x: torch.Tensor,
                       row_sigma: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
        """x [..., 24] -> (shape index int64, gain index int32).  row_sigma
        (broadcast to x[..., 0]) divides the gain before coding, e.g. per
        weight row.  One library call: search, ranking and gain code."""
        idx, gain = self._run(x, row_sigma, pack=False)
        return idx, gain

    def _run(self, x: torch.Tensor, row_sigma: torch.Tensor | None, pack: bool):
        from . import _native

        dev = self.shape.device
        if dev.type != "cuda":
            raise ValueError("shape-gain quantization requires a CUDA device")
        x = torch.as_tensor(x, dtype=torch.float32, device=dev)
        if x.shape[-1] != DIM:
            raise ValueError(f"expected last dimension {DIM}, got {x.shape[-1]}")
        shape = x.shape[:-1]
        xs = x.reshape(-1, DIM).contiguous()
        n = xs.shape[0]
        idx = torch.empty(n, dtype=torch.long, device=dev)
        pair = torch.empty(n, dtype=torch.long, device=dev)
        score = torch.empty(n, dtype=torch.float32, device=dev)
        gain = None if pack else torch.empty(n, dtype=torch.int32, device=dev)
        sig = None
        if row_sigma is not None:
            sig = torch.broadcast_to(torch.as_tensor(row_sigma, dtype=torch.float32, device=dev),
                                     shape).reshape(-1).contiguous()
        with torch.cuda.device(dev):
            self.shape._book().quantize_gain(
                xs.data_ptr(), n, idx.data_ptr(), pair.data_ptr(), score.data_ptr(), self.thresholds.data_ptr(),
                self.gain_bits, sig.data_ptr() if sig is not None else None, 1,
                gain.data_ptr() if gain is not None else None, pack, torch.cuda.current_stream().cuda_stream,
                angular=self.multi_shell)
        return idx.reshape(shape), (gain.reshape(shape) if gain is not None else None)

    def dequantize_parts(self, sidx: torch.Tensor, gidx: torch.Tensor,
                         row_sigma: torch.Tensor | None = None) -> torch.Tensor:
        g = self.levels[gidx.to(device=self.shape.device, dtype=torch.long)]
        if row_sigma is not None:
            g = g * row_sigma
        v = self.shape.dequantize(sidx.to(self.shape.device))
        if self.multi_shell:  # |y| / sqrt(8) = sqrt(2 shell) varies with the shell
            return v * (g / v.norm(dim=-1)).unsqueeze(-1)
        return v * (g / self.norm).unsqueeze(-1)

    def quantize(self, x: torch.Tensor, row_sigma: torch.Tensor | None = None) -> torch.Tensor:
        """x [..., 24] -> combined int64 indices shape * 2^b + gain.  Rates
        whose index exceeds 63 bits (3.0 bits/dim: 62 + 10) raise ValueError;
        use quantize_parts for them."""
        self._check_packable()
        return self._run(x, row_sigma, pack=True)[0]

    def dequantize(self, indices: torch.Tensor, row_sigma: torch.Tensor | None = None) -> torch.Tensor:
        self._check_packable()
        indices = indices.to(self.shape.device)
        return self.dequantize_parts(indices >> self.gain_bits, indices & ((1 << self.gain_bits) - 1), row_sigma)

    def _check_packable(self) -> None:
        if self.bits > 63:
            raise ValueError(f"a {self.bits}-bit shape-gain index does not fit int64; use quantize_parts / "
                             "dequantize_parts")
