"""GPU tests of the DLRM dense tower (include/xse_dlrm.h): Dense layers and the
strided dot interaction against float64 references on the host, then the
whole forward (pooled lookup + tower) against the oracle's pooling followed by
the float64 tower. Floating-point tolerances: Dense layers 1e-5 relative to
the magnitude sum sum_i |x_i k_i| + |b| (fp32 GEMM, any summation order);
interaction 1e-4 relative to sum_c |z_i,c z_j,c|; predictions 1e-4
absolute (sigmoid outputs in (0, 1))."""

import numpy as np
import pytest
import torch

from oracle import oracle

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dlrm(xse):
  from xla_serving_b200 import dlrm as dlrm_module  # pylint: disable=import-outside-toplevel
  return dlrm_module


def host_linear(x, kernel, bias, act):
  y = x.astype(np.float64) @ kernel.astype(np.float64)
  if bias is not None:
    y += bias
  if act == 1:
    y = np.maximum(y, 0.0)
  elif act == 2:
    y = 1.0 / (1.0 + np.exp(-y))
  bound = np.abs(x.astype(np.float64)) @ np.abs(kernel.astype(np.float64))
  if bias is not None:
    bound += np.abs(bias)
  return y, bound


@pytest.mark.parametrize("rows,in_dim,out_dim,x_pad,y_pad,act,with_bias", [
    (64, 13, 512, 0, 0, 1, True),      # bottom MLP input layer (K = 13)
    (100, 479, 1024, 1, 0, 1, True),   # top MLP input from a padded row
    (37, 256, 1, 0, 0, 2, True),       # sigmoid head (own kernel)
    (50, 64, 33, 3, 5, 0, False),      # no bias, no activation, strided
    (20, 32, 7, 0, 2, 2, True),        # sigmoid on a wide output
    (1, 128, 256, 0, 0, 1, True),      # single row
])
def test_linear_forward(xse, rows, in_dim, out_dim, x_pad, y_pad, act,
                        with_bias):
  rng = np.random.default_rng(rows * 1000 + in_dim + out_dim)
  x_full = rng.standard_normal((rows, in_dim + x_pad)).astype(np.float32)
  kernel = rng.uniform(-0.2, 0.2, (in_dim, out_dim)).astype(np.float32)
  bias = (rng.uniform(-0.1, 0.1, out_dim).astype(np.float32)
          if with_bias else None)
  x_dev = torch.from_numpy(x_full).cuda()
  k_dev = torch.from_numpy(kernel).cuda()
  b_dev = torch.from_numpy(bias).cuda() if with_bias else None
  y_dev = torch.full((rows, out_dim + y_pad), 7.0, device="cuda")
  C = xse._capi
  C.check(C.lib.xse_linear_forward(
      x_dev.data_ptr(), rows, in_dim, x_dev.stride(0), k_dev.data_ptr(),
      None if b_dev is None else b_dev.data_ptr(), out_dim, act, C.MATH_FP32,
      y_dev.data_ptr(), y_dev.stride(0), None))
  torch.cuda.synchronize()
  got = y_dev.cpu().numpy()
  want, bound = host_linear(x_full[:, :in_dim], kernel, bias, act)
  np.testing.assert_array_less(np.abs(got[:, :out_dim] - want),
                               1e-5 * bound + 1e-6)
  if y_pad:
    assert np.all(got[:, out_dim:] == 7.0)  # untouched padding


def test_linear_forward_errors(xse):
  C = xse._capi
  rc = C.lib.xse_linear_forward(None, 4, 8, 4, None, None, 2, 1, 0, None, 2,
                                None)
  assert rc == C.INVALID_ARGUMENT and "strides" in C.last_error()
  rc = C.lib.xse_linear_forward(None, 4, 8, 8, None, None, 2, 9, 0, None, 2,
                                None)
  assert rc == C.INVALID_ARGUMENT and "activation" in C.last_error()
  rc = C.lib.xse_linear_forward(None, 4, 8, 8, None, None, 2, 1, 7, None, 2,
                                None)
  assert rc == C.INVALID_ARGUMENT and "math" in C.last_error()
  assert C.lib.xse_linear_forward(None, 0, 8, 8, None, None, 2, 1, 0, None, 2,
                                  None) == C.OK


@pytest.mark.parametrize("batch,tables,dim,out_pad", [
    (333, 26, 128, 1), (64, 26, 128, 9), (50, 3, 24, 4), (9, 5, 7, 0)])
def test_dot_interaction_strided(xse, batch, tables, dim, out_pad):
  rng = np.random.default_rng(batch + tables)
  dense_full = rng.standard_normal((batch, dim + 4)).astype(np.float32)
  pooled_full = rng.standard_normal((batch, tables * dim + 8)).astype(
      np.float32)
  width = dim + (tables + 1) * tables // 2
  dense = torch.from_numpy(dense_full).cuda()
  pooled = torch.from_numpy(pooled_full).cuda()
  out = torch.full((batch, width + out_pad), 3.0, device="cuda")
  C = xse._capi
  C.check(C.lib.xse_dot_interaction_strided(
      dense.data_ptr(), dense.stride(0), pooled.data_ptr(), pooled.stride(0),
      batch, tables, dim, out.data_ptr(), out.stride(0), None))
  torch.cuda.synchronize()
  got = out.cpu().numpy()
  d = dense_full[:, :dim]
  p = pooled_full[:, :tables * dim].reshape(batch, tables, dim)
  want = oracle.dot_interaction(d, p)
  z = np.concatenate([d[:, None, :], p], axis=1).astype(np.float64)
  mag = np.abs(z) @ np.abs(z).transpose(0, 2, 1)
  iu = np.triu_indices(tables + 1, 1)
  bound = np.concatenate([np.abs(d), mag[:, iu[0], iu[1]]], axis=1)
  np.testing.assert_array_less(np.abs(got[:, :width] - want),
                               1e-4 * bound + 1e-7)
  np.testing.assert_array_equal(got[:, :dim], d)  # dense part copied as is
  assert np.all(got[:, width:] == 0.0)  # padding zeroed


def test_dot_interaction_strided_rejects_short_strides(xse):
  C = xse._capi
  rc = C.lib.xse_dot_interaction_strided(None, 127, None, 26 * 128, 1, 26,
                                         128, None, 479, None)
  assert rc == C.INVALID_ARGUMENT and "strides" in C.last_error()


@pytest.mark.parametrize("math", ["fp32", "tf32x3"])
def test_dense_tower_matches_float64(xse, dlrm, math):
  code = xse._capi.MATH_FP32 if math == "fp32" else dlrm.MATH_TF32X3
  tower = dlrm.DenseTower(seed=3, math=code)
  rng = np.random.default_rng(5)
  batch = 96
  dense = rng.standard_normal((batch, 13)).astype(np.float32)
  pooled = rng.uniform(-1, 1, (batch, 26, 128)).astype(np.float32)
  got = tower.forward(torch.from_numpy(dense).cuda(),
                      torch.from_numpy(pooled).cuda()).cpu().numpy()
  want = tower.reference_forward(dense, pooled)
  assert got.shape == (batch,)
  np.testing.assert_allclose(got, want, rtol=0, atol=1e-4)
  assert np.all((got > 0) & (got < 1))


@pytest.mark.parametrize("rows,in_dim,out_dim,act", [
    (300, 480, 1024, 1), (77, 1024, 512, 1), (64, 256, 128, 0),
    (1, 128, 256, 1)])
def test_linear_forward_tf32x3(xse, dlrm, rows, in_dim, out_dim, act):
  """Three TF32 GEMMs over split operands: fp32-level accuracy (the same
  1e-5 magnitude-relative bound as the fp32 layer)."""
  rng = np.random.default_rng(rows + in_dim)
  x = rng.standard_normal((rows, in_dim)).astype(np.float32)
  kernel = rng.uniform(-0.1, 0.1, (in_dim, out_dim)).astype(np.float32)
  bias = rng.uniform(-0.1, 0.1, out_dim).astype(np.float32)
  xd, kd = torch.from_numpy(x).cuda(), torch.from_numpy(kernel).cuda()
  xh, xl = torch.empty_like(xd), torch.empty_like(xd)
  kh, kl = torch.empty_like(kd), torch.empty_like(kd)
  dlrm.tf32_split(xd, xh, xl)
  dlrm.tf32_split(kd, kh, kl)
  # the split is exact and hi has at most 11 significant bits
  torch.testing.assert_close(xh + xl, xd, rtol=0, atol=0)
  assert torch.all((xh.view(torch.int32) & 0x1FFF) == 0)
  layer = dlrm.DenseLayer(kd, torch.from_numpy(bias).cuda(), act)
  out = torch.empty((rows, out_dim), device="cuda")
  dlrm.linear_tf32x3(xh, xl, kh, kl, layer, out)
  torch.cuda.synchronize()
  want, bound = host_linear(x, kernel, bias, act)
  np.testing.assert_array_less(np.abs(out.cpu().numpy() - want),
                               1e-5 * bound + 1e-6)


@pytest.mark.parametrize("fused_interaction,math,index", [
    (False, "fp32", "i64"), (True, "fp32", "i64"), (True, "tf32x3", "i32"),
    (False, "tf32x3", "i32")])
def test_dlrm_forward_end_to_end(xse, dlrm, fused_interaction, math, index):
  """Pooled lookup of 26 fp32 features (ragged Zipf bags, sum pooling) plus
  the tower: pooled values bit-exact to the oracle (unfused: read back from
  the pooled buffer), predictions within 1e-4 of the float64 tower applied to
  the oracle's pooled values (fused: pooling and interaction in one
  kernel, the pooled rows never stored; fused split-TF32: the interaction
  kernel writes the first top layer's split operands). Ids and row pointers
  int64, or int32 as the reference's DLRM bundle feeds them."""
  from xla_serving_b200 import synth  # pylint: disable=import-outside-toplevel
  engine = xse.EmbeddingEngine()
  rows = synth.log_uniform_rows(26, 50, 5000, 7)
  names, host_tables = [], []
  ids, offsets = [], []
  batch = 128
  for t in range(26):
    table, _, _ = synth.synth_table(xse._capi.DT_F32, rows[t], 128, 11, t)
    name = f"sparse_{t}"
    engine.add_table(name, table, "SUM")
    engine.register_feature(name, name)
    names.append(name)
    host_tables.append(table.cpu().numpy())
    spec = synth.TableSpec(name, rows[t], 128, xse._capi.DT_F32, "SUM")
    fb = synth.synth_batch(spec, t, batch, 1, 100, 11, 1.05)
    idt = torch.int32 if index == "i32" else torch.int64
    ids.append(fb.ids.to(idt))
    offsets.append(fb.offsets.to(idt))
  model = dlrm.DLRM(engine, names, seed=1,
                    fused_interaction=fused_interaction,
                    math=dlrm.MATH_TF32X3 if math == "tf32x3"
                    else xse._capi.MATH_FP32)
  dense = torch.randn(batch, 13, generator=torch.Generator().manual_seed(2))
  pred = model.forward(dense.cuda(), ids, offsets).cpu().numpy()
  pooled = np.stack([
      oracle.embedding_bag(host_tables[t], ids[t].cpu().numpy(),
                           offsets[t].cpu().numpy(), None, "SUM")
      for t in range(26)], axis=1)
  if not fused_interaction:
    np.testing.assert_array_equal(model.pooled_buffer(batch).cpu().numpy(),
                                  pooled)
  want = model.tower.reference_forward(dense.numpy(), pooled)
  np.testing.assert_allclose(pred, want, rtol=0, atol=1e-4)
  engine.close()


@pytest.mark.parametrize("dim,tables", [(128, 26), (64, 5)])
def test_interaction_split_operands(xse, dim, tables):
  """execute_interaction with out_lo writes the values' TF32 parts and the
  exact remainders: hi + lo equals the plain call's values bit for bit, hi
  has no bits below TF32 precision and |lo| <= 2^-11 |value|. dim 128 fp32
  runs the fused kernel, dim 64 the pooling + interaction fallback."""
  rng = np.random.default_rng(dim + tables)
  engine = xse.EmbeddingEngine()
  batch = 96
  reqs = []
  for t in range(tables):
    table = torch.from_numpy(
        rng.uniform(-1, 1, (300, dim)).astype(np.float32)).cuda()
    engine.add_table(f"t{t}", table, "SUM")
    engine.register_feature(f"f{t}", f"t{t}")
    lengths = rng.integers(0, 9, batch)
    offsets = np.concatenate([[0], np.cumsum(lengths)])
    ids = rng.integers(0, 300, int(offsets[-1]))
    reqs.append(xse.BagRequest(f"f{t}", torch.from_numpy(ids).cuda(),
                               torch.from_numpy(offsets).cuda(), None))
  dense = torch.randn(batch, dim, device="cuda")
  width = dim + (tables + 1) * tables // 2
  stride = (width + 3) // 4 * 4 + 4
  plain = torch.full((batch, stride), 9.0, device="cuda")
  engine.execute_interaction(reqs, dense, plain, fused=True)
  hi = torch.full_like(plain, 7.0)
  lo = torch.full_like(plain, 7.0)
  engine.execute_interaction(reqs, dense, hi, fused=True, out_lo=lo)
  v = plain.cpu().numpy()
  h = hi.cpu().numpy()
  l = lo.cpu().numpy()
  np.testing.assert_array_equal((h + l).view(np.uint32), v.view(np.uint32))
  assert not (h.view(np.uint32) & 0x1fff).any()
  assert (np.abs(l) <= np.abs(v) * 2.0 ** -11).all()
  engine.close()
