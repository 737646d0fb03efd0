"""Shared helpers of the GPU parity tests: build the same request on the
engine (CUDA, through the C ABI) and on the oracle (CPU), compare."""

import numpy as np
import torch

from oracle import oracle

TORCH_DT = {oracle.F32: torch.float32, oracle.BF16: torch.bfloat16,
            oracle.I8_ROWWISE: torch.int8}


def random_table(rng, dtype, vocab, dim):
  """Returns (host table in oracle layout, device tensor, scale, bias)."""
  if dtype == oracle.F32:
    host = rng.uniform(-1, 1, (vocab, dim)).astype(np.float32)
    return host, torch.from_numpy(host).cuda(), None, None
  if dtype == oracle.BF16:
    f = rng.uniform(-1, 1, (vocab, dim)).astype(np.float32)
    bits = (f.view(np.uint32) >> 16).astype(np.uint16)
    dev = torch.from_numpy(bits.view(np.int16)).cuda().view(torch.bfloat16)
    return bits, dev, None, None
  q = rng.integers(-127, 128, (vocab, dim)).astype(np.int8)
  scale = rng.uniform(1e-3, 1e-2, vocab).astype(np.float32)
  bias = rng.uniform(-0.1, 0.1, vocab).astype(np.float32)
  return q, torch.from_numpy(q).cuda(), scale, bias


def random_csr(rng, vocab, bags, max_len, first=0, empty_frac=0.1):
  lengths = rng.integers(0, max_len + 1, bags)
  lengths[rng.random(bags) < empty_frac] = 0
  offsets = np.concatenate([[first], first + np.cumsum(lengths)])
  ids = rng.integers(0, vocab, int(offsets[-1]))
  # Positions before the first offset are never read or validated
  # (absolute CSR offsets, embedding_bag.cc:110-133): make them invalid.
  ids[:first] = -7
  return ids.astype(np.int64), offsets.astype(np.int64)


def to_dev(a, dtype=None):
  t = torch.from_numpy(np.ascontiguousarray(a))
  if dtype is not None:
    t = t.to(dtype)
  return t.cuda()


def oracle_pool(host_table, dtype, ids, offsets, weights, combine, scale=None,
                bias=None):
  return oracle.embedding_bag(host_table, ids, offsets, weights, combine,
                              dtype, scale, bias, num_threads=4)


# Int8 row-wise tables: the oracle states the dequantization as an fp32 row
# (float(q) * scale rounded, then + bias rounded) pooled in fp32; the kernel
# dequantizes each element with one fma (one rounding). Results are compared
# within INT8_RTOL of the condition-aware bound sum_i |w_i| (|q_i| s_i +
# |b_i|) per output element (the same bag pooled over absolute values), so a
# sum that cancels to near zero is not held to a relative bound it cannot
# meet. Both roundings are within 2^-24 of that bound per term.
INT8_RTOL = 1e-5


def int8_bound(host_table, ids, offsets, weights, combine, scale, bias):
  """sum |w| (|q| scale + |bias|) per output element, with the bag's mean or
  sqrt-n factor (computed by the oracle over absolute values)."""
  return oracle.embedding_bag(
      np.abs(host_table.astype(np.int16)).astype(np.int8), ids, offsets,
      None if weights is None else np.abs(weights), combine,
      oracle.I8_ROWWISE, np.abs(scale), np.abs(bias), num_threads=4)


def expect_pool(host_table, dtype, ids, offsets, weights, combine, scale=None,
                bias=None):
  """The oracle's pooled output, and for int8 tables the bound that the
  comparison scales its tolerance by (None: bit-exact)."""
  want = oracle_pool(host_table, dtype, ids, offsets, weights, combine, scale,
                     bias)
  bound = None
  if dtype == oracle.I8_ROWWISE:
    bound = int8_bound(host_table, ids, offsets, weights, combine, scale,
                       bias)
  return want, bound


def assert_pooled(got, expected, what=""):
  """Compares with expect_pool's result: bit for bit, or for int8 tables
  |got - want| <= INT8_RTOL * bound."""
  want, bound = expected
  if bound is None:
    assert_bitwise(got, want, what)
    return
  got = np.asarray(got, dtype=np.float64)
  want = np.asarray(want, dtype=np.float64)
  assert got.shape == want.shape, (what, got.shape, want.shape)
  err = np.abs(got - want)
  lim = INT8_RTOL * np.asarray(bound, dtype=np.float64)
  bad = err > lim
  if bad.any():
    idx = np.argwhere(bad)[:5]
    k = tuple(idx[0])
    raise AssertionError(
        f"{what}: {int(bad.sum())} of {got.size} beyond {INT8_RTOL} x bound, "
        f"first at {idx.tolist()}: got {got[k]} want {want[k]} bound "
        f"{bound[k]}; max abs err {err.max():.3g}")


def assert_bitwise(got, want, what=""):
  got = np.asarray(got, dtype=np.float32)
  want = np.asarray(want, dtype=np.float32)
  assert got.shape == want.shape, (what, got.shape, want.shape)
  same = (got.view(np.uint32) == want.view(np.uint32)) | (
      np.isnan(got) & np.isnan(want))
  if not same.all():
    idx = np.argwhere(~same)[:5]
    raise AssertionError(
        f"{what}: {int((~same).sum())} of {got.size} differ, first at "
        f"{idx.tolist()}: got {got[tuple(idx[0])]} want {want[tuple(idx[0])]}")
