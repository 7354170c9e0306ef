"""Seeded synthetic workloads with the shapes of the hot path's benchmark configs.

All inputs are synthetic (the reference publishes no dataset): keys are the
SplitMix64 sequence, hot-key skew is a Zipf law over a seeded permutation of
the warmed keys, gradients are Gaussian.

  splitmix64_sequence(i) = fmix64((i + 1) * 0x9e3779b97f4a7c15 mod 2^64),
  the i-th output of the SplitMix64 generator seeded with 0 (a bijection of i).
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np

GOLDEN = np.uint64(0x9E3779B97F4A7C15)


def fmix64(z: np.ndarray) -> np.ndarray:
    z = np.asarray(z, dtype=np.uint64).copy()
    with np.errstate(over="ignore"):
        z ^= z >> np.uint64(30)
        z *= np.uint64(0xBF58476D1CE4E5B9)
        z ^= z >> np.uint64(27)
        z *= np.uint64(0x94D049BB133111EB)
        z ^= z >> np.uint64(31)
    return z


def splitmix64_sequence(idx) -> np.ndarray:
    i = np.asarray(idx, dtype=np.uint64)
    with np.errstate(over="ignore"):
        return fmix64((i + np.uint64(1)) * GOLDEN)


class Zipf:
    """Inverse-CDF sampler of ranks 1..n with weights r^-alpha, mapped through
    a seeded permutation so hot items are scattered over the key space."""

    def __init__(self, n: int, alpha: float, seed: int):
        w = np.arange(1, n + 1, dtype=np.float64) ** (-alpha)
        self.cdf = np.cumsum(w)
        self.cdf /= self.cdf[-1]
        self.perm = np.random.default_rng(seed).permutation(n)

    def sample(self, rng: np.random.Generator, size: int) -> np.ndarray:
        u = rng.random(size)
        r = np.searchsorted(self.cdf, u, side="right")
        r = np.minimum(r, len(self.cdf) - 1)
        return self.perm[r]


@dataclass
class ForwardWorkload:
    """Forward-only lookup: dim-32 fp32 store warmed with `num_keys`
    splitmix64 keys; batches of `batch` keys Zipf(alpha) over them."""

    num_keys: int = 1_000_000
    dim: int = 32
    batch: int = 4096
    alpha: float = 1.1
    seed: int = 0x5EED5CA1E

    def warm_keys(self) -> np.ndarray:
        return splitmix64_sequence(np.arange(self.num_keys))

    def batches(self, count: int) -> np.ndarray:
        z = Zipf(self.num_keys, self.alpha, self.seed)
        rng = np.random.default_rng(self.seed)
        idx = z.sample(rng, count * self.batch).reshape(count, self.batch)
        return splitmix64_sequence(idx)


@dataclass
class TrainWorkload:
    """Single-table train step: dim-64 fp32, `num_keys` warmed int64 keys;
    batches of `batch` keys, (1 - new_fraction) Zipf(alpha) over the warmed
    keys and new_fraction never-seen keys inserted on miss; gradients
    N(0, sigma) with sigma = 1e-3 (standard deviation)."""

    num_keys: int = 10_000_000
    dim: int = 64
    batch: int = 65536
    alpha: float = 1.05
    new_fraction: float = 0.05
    sigma: float = 1e-3
    seed: int = 0xC0FFEE
    rank: int = 0

    def warm_keys(self) -> np.ndarray:
        return splitmix64_sequence(np.arange(self.num_keys)).view(np.int64)

    def make_batches(self, count: int, start_step: int = 0):
        """(keys[count, batch] int64, grads[count, batch, dim] float32)."""
        z = Zipf(self.num_keys, self.alpha, self.seed)
        rng = np.random.default_rng([self.seed, self.rank, start_step])
        n_new = int(round(self.batch * self.new_fraction))
        n_old = self.batch - n_new
        keys = np.empty((count, self.batch), dtype=np.int64)
        for s in range(count):
            old = splitmix64_sequence(z.sample(rng, n_old))
            base = self.num_keys + ((start_step + s) * 1024 + self.rank) * n_new
            new = splitmix64_sequence(np.arange(base, base + n_new, dtype=np.uint64))
            k = np.concatenate([old, new])
            rng.shuffle(k)
            keys[s] = k.view(np.int64)
        grads = (rng.standard_normal((count, self.batch, self.dim), dtype=np.float32) * np.float32(self.sigma))
        return keys, grads


@dataclass
class DlrmWorkload:
    """DLRM-style multi-table step: `tables` tables with row counts
    log-uniform in [min_rows, max_rows] (seeded), dim 128; per sample and
    table max(1, Poisson(mean_ids)) ids drawn Zipf(alpha) over the table's
    rows. A key is fmix64((table << 40) | id): a pre-mixed u64, so every
    partitioner spreads the tables over the GPUs. The harness sum-pools the
    rows of each (sample, table) and broadcasts a N(0, sigma) pooled
    gradient back to each of its ids."""

    tables: int = 26
    min_rows: int = 1_000
    max_rows: int = 40_000_000
    dim: int = 128
    batch: int = 8192
    mean_ids: float = 20.0
    alpha: float = 1.2
    sigma: float = 1e-3
    seed: int = 0xD1A
    rank: int = 0

    def table_rows(self) -> np.ndarray:
        rng = np.random.default_rng(self.seed)
        lo, hi = np.log(self.min_rows), np.log(self.max_rows)
        return np.round(np.exp(rng.uniform(lo, hi, size=self.tables))).astype(np.int64)

    def make_batch(self, step: int):
        """(keys u64 [n], bag [n] int64 = sample * tables + table, pooled grads
        [batch * tables, dim] float32) for one step."""
        rows = self.table_rows()
        rng = np.random.default_rng([self.seed, self.rank, step])
        keys, bags = [], []
        for t in range(self.tables):
            z = Zipf(int(rows[t]), self.alpha, self.seed + t)
            counts = np.maximum(1, rng.poisson(self.mean_ids, size=self.batch))
            ids = z.sample(rng, int(counts.sum())).astype(np.uint64)
            keys.append(fmix64((np.uint64(t) << np.uint64(40)) | ids))
            bags.append(np.repeat(np.arange(self.batch, dtype=np.int64) * self.tables + t, counts))
        pooled = rng.standard_normal((self.batch * self.tables, self.dim), dtype=np.float32) * np.float32(self.sigma)
        return np.concatenate(keys), np.concatenate(bags), pooled

    def make_bags(self, step: int):
        """The same batch grouped by bag: (keys u64 [n] ordered by bag, each
        bag's ids in draw order; offsets int64 [batch * tables + 1]; pooled
        grads [batch * tables, dim] float32)."""
        keys, bag, pooled = self.make_batch(step)
        order = np.argsort(bag, kind="stable")
        offsets = np.zeros(self.batch * self.tables + 1, dtype=np.int64)
        offsets[1:] = np.cumsum(np.bincount(bag, minlength=self.batch * self.tables))
        return keys[order], offsets, pooled

    def device_bags(self, step: int, torch, device="cuda"):
        """One batch grouped by bag, generated on the device (the stated row
        ranges up to 4e7 per table without host-side samplers): (keys uint64
        [n] ordered by bag = sample * tables + table; offsets int64
        [batch * tables + 1]; bag of each id int64 [n]; pooled grads
        [batch * tables, dim] float32). Same laws as make_bags, other draws:
        counts max(1, Poisson(mean_ids)); the Zipf(alpha) rank of an id by the
        continuous inverse CDF over the table's rows n_t,
        rank = ((n_t^(1-a) - 1) u + 1)^(1/(1-a)), and the rank goes to row
        fmix64((t << 40) | rank) mod n_t, which scatters each table's hot
        rows without a stored permutation."""
        gen = torch.Generator(device=device).manual_seed((self.seed << 24) ^ (step << 8) ^ self.rank)
        T, B = self.tables, self.batch
        rows = torch.as_tensor(self.table_rows(), dtype=torch.int64, device=device)
        lam = torch.full((B, T), float(self.mean_ids), dtype=torch.float32, device=device)
        counts = torch.poisson(lam, generator=gen).to(torch.int64).clamp_(min=1).reshape(-1)
        offsets = torch.zeros(B * T + 1, dtype=torch.int64, device=device)
        torch.cumsum(counts, 0, out=offsets[1:])
        bag = torch.repeat_interleave(torch.arange(B * T, dtype=torch.int64, device=device), counts)
        table = bag % T
        n_t = rows[table]
        u = torch.rand(bag.numel(), generator=gen, device=device, dtype=torch.float64)
        a1 = 1.0 - self.alpha
        r = (((n_t.to(torch.float64) ** a1 - 1.0) * u + 1.0) ** (1.0 / a1)).floor()
        rank = torch.minimum(r.to(torch.int64), n_t).clamp_(min=1) - 1
        mixed = CapacityWorkload._fmix64_t((table << 40) | rank)
        ids = (mixed & 0x7FFFFFFFFFFFFFFF) % n_t
        keys = CapacityWorkload._fmix64_t((table << 40) | ids)
        pooled = torch.randn((B * T, self.dim), generator=gen, device=device) * self.sigma
        return keys.view(torch.uint64), offsets, bag, pooled

    @staticmethod
    def encode_keys_like(ids, table: int, slot_bits: int = 16):
        """The reference's encode_keys layout, (table << (64 - slot_bits)) |
        (id & mask), on an int64 tensor of raw ids (returned as int64 bit
        patterns): the table-prefixed keys that fast_range sends to one
        shard."""
        mask = (1 << (64 - slot_bits)) - 1
        prefix = table << (64 - slot_bits)
        if prefix >= 1 << 63:
            prefix -= 1 << 64
        return (ids & mask) | prefix


@dataclass
class CapacityWorkload:
    """Capacity run: `num_keys` u64 keys splitmix64(i), dim 64 fp32 with Adam
    state; batches of `batch` keys, (1 - new_fraction) Zipf(alpha) over the
    keys and new_fraction never-seen keys; gradients N(0, sigma). On g GPUs,
    rank r warms the keys the partitioner maps to r."""

    num_keys: int = 1_500_000_000
    dim: int = 64
    batch: int = 262_144
    alpha: float = 1.05
    new_fraction: float = 0.01
    sigma: float = 1e-3
    seed: int = 0xCA9
    rank: int = 0

    def warm_keys(self) -> np.ndarray:
        return splitmix64_sequence(np.arange(self.num_keys))

    def make_batches(self, count: int, start_step: int = 0):
        z = Zipf(self.num_keys, self.alpha, self.seed)
        rng = np.random.default_rng([self.seed, self.rank, start_step])
        n_new = int(round(self.batch * self.new_fraction))
        keys = np.empty((count, self.batch), dtype=np.uint64)
        for s in range(count):
            old = splitmix64_sequence(z.sample(rng, self.batch - n_new))
            base = self.num_keys + ((start_step + s) * 1024 + self.rank) * n_new
            new = splitmix64_sequence(np.arange(base, base + n_new, dtype=np.uint64))
            k = np.concatenate([old, new])
            rng.shuffle(k)
            keys[s] = k
        grads = rng.standard_normal((count, self.batch, self.dim), dtype=np.float32) * np.float32(self.sigma)
        return keys, grads


    # ---- on-device generation (the stated scale: no host copy of 1.5e9 keys) ----
    # torch has no unsigned 64-bit arithmetic for these ops, so the keys are
    # computed on int64 tensors holding the u64 bit patterns (multiplication
    # wraps mod 2^64; right shifts are made logical by masking).

    @staticmethod
    def _lsr(z, k: int):
        return (z >> k) & ((1 << (64 - k)) - 1)

    @classmethod
    def _fmix64_t(cls, z):
        z = z ^ cls._lsr(z, 30)
        z = z * _I64_C1
        z = z ^ cls._lsr(z, 27)
        z = z * _I64_C2
        return z ^ cls._lsr(z, 31)

    @classmethod
    def splitmix64_t(cls, idx):
        """splitmix64_sequence of an int64 index tensor, as int64 bit patterns."""
        return cls._fmix64_t((idx + 1) * _I64_GOLDEN)

    def device_keys(self, start: int, count: int, torch, device="cuda"):
        """Keys splitmix64(i) for i in [start, start + count), uint64 on the device."""
        i = torch.arange(start, start + count, dtype=torch.int64, device=device)
        return self.splitmix64_t(i).view(torch.uint64)

    def device_batch(self, step: int, torch, device="cuda"):
        """One batch on the device: (1 - new_fraction) Zipf(alpha) draws over
        the keys and new_fraction never-seen keys, uint64; gradients
        N(0, sigma) fp32. The Zipf law at this scale is sampled by the
        continuous inverse CDF, rank = ((n^(1-a) - 1) u + 1)^(1/(1-a)), and
        a rank goes to item fmix64(rank) mod n, which scatters the hot ranks
        over the key space without a stored permutation."""
        gen = torch.Generator(device=device).manual_seed((self.seed << 20) ^ (step << 8) ^ self.rank)
        n_new = int(round(self.batch * self.new_fraction))
        n_old = self.batch - n_new
        u = torch.rand(n_old, generator=gen, device=device, dtype=torch.float64)
        a1 = 1.0 - self.alpha
        r = (((float(self.num_keys) ** a1 - 1.0) * u + 1.0) ** (1.0 / a1)).floor().clamp_(1, self.num_keys)
        rank = r.to(torch.int64) - 1
        item = (self._fmix64_t(rank) & 0x7FFFFFFFFFFFFFFF) % self.num_keys
        base = self.num_keys + (step * 1024 + self.rank) * n_new
        new = torch.arange(base, base + n_new, dtype=torch.int64, device=device)
        keys = self.splitmix64_t(torch.cat([item, new]))
        keys = keys[torch.randperm(self.batch, generator=gen, device=device)]
        grads = torch.randn((self.batch, self.dim), generator=gen, device=device) * self.sigma
        return keys.view(torch.uint64), grads


_I64_GOLDEN = int(np.int64(np.uint64(0x9E3779B97F4A7C15).view(np.int64)))
_I64_C1 = int(np.uint64(0xBF58476D1CE4E5B9).view(np.int64))
_I64_C2 = int(np.uint64(0x94D049BB133111EB).view(np.int64))


@dataclass
class InferenceWorkload:
    """Weight-only inference store: int32 keys 0 .. num_keys-1, dim 256
    bf16 values from the Uniform(-0.05, 0.05) initializer, no optimizer;
    forward_lookup batches of `batch` keys uniform over the key set."""

    num_keys: int = 200_000_000
    dim: int = 256
    batch: int = 262_144
    seed: int = 0x1BF

    def warm_keys(self) -> np.ndarray:
        return np.arange(self.num_keys, dtype=np.int32)

    def batches(self, count: int, start: int = 0) -> np.ndarray:
        rng = np.random.default_rng([self.seed, start])
        return rng.integers(0, self.num_keys, size=(count, self.batch), dtype=np.int32)
