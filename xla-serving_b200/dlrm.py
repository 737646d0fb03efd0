"""DLRM forward pass on the B200.

The reference's DLRM bundle pools its 26 sparse features through
CpuEmbeddingLookupTransform and feeds them, with 13 dense features, to a
dense tower under XLA (examples/dlrm/model_jce.py:98-189): bottom MLP
13-512-256-128 with ReLU, feature interaction over the 27 vectors, top MLP
1024-1024-512-256-1 with a sigmoid head. Here every stage runs on the device:
the pooled lookup in the engine's kernels, the dot interaction (27 x 27
Gram, upper triangle, dense output first: 128 + 351 = 479 features) in place
of the reference's DCN-v2 cross network, and the Dense layers with fused
bias+ReLU (xse_linear_forward): fp32 GEMMs, or -- MATH_TF32X3, what the
benchmark runs -- three TF32 tensor-core GEMMs over hi/lo split operands
(fp32-level accuracy). With the fused interaction the interaction kernel
writes the first top layer's split operands itself.

Initialisation: Dense kernels Xavier-uniform, biases U(-1/sqrt(fan_in),
1/sqrt(fan_in)) as the reference's uniform_init (model_jce.py:107-118),
drawn from numpy's default_rng(seed).
"""

import dataclasses
from typing import List, Optional, Sequence

import numpy as np
import torch

from . import _capi as C
from .engine import BagRequest, EmbeddingEngine, Status, stream_handle

BOTTOM_MLP = (512, 256, 128)
TOP_MLP = (1024, 1024, 512, 256, 1)
# Dense-layer arithmetic of the tower: C.MATH_FP32 (CUDA-core fp32 GEMMs),
# C.MATH_TF32 (one TF32 GEMM: reduced precision), or MATH_TF32X3 (three TF32
# tensor-core GEMMs over hi/lo split operands: fp32-level accuracy).
MATH_TF32X3 = 3


def interaction_width(num_tables, dim):
  rows = num_tables + 1
  return dim + rows * (rows - 1) // 2


def _round_up(x, m):
  return (x + m - 1) // m * m


@dataclasses.dataclass
class DenseLayer:
  kernel: torch.Tensor  # [in, out] fp32, flax.linen.Dense layout
  bias: torch.Tensor    # [out] fp32
  activation: int


def init_dense_layers(in_dim, dims, rng, last_sigmoid):
  """Dense layers in_dim -> dims[0] -> ... with ReLU (sigmoid on the last
  layer when last_sigmoid), as numpy arrays (kernel [in, out], bias)."""
  layers = []
  prev = in_dim
  for k, out in enumerate(dims):
    bound = np.sqrt(6.0 / (prev + out))
    kernel = rng.uniform(-bound, bound, (prev, out)).astype(np.float32)
    b = np.sqrt(1.0 / prev)
    bias = rng.uniform(-b, b, out).astype(np.float32)
    last = k == len(dims) - 1
    act = C.ACT_SIGMOID if (last and last_sigmoid) else C.ACT_RELU
    layers.append((kernel, bias, act))
    prev = out
  return layers


def tf32_split(x, hi, lo, stream=None):
  """hi = x rounded to TF32, lo = x - hi (2-D tensors of x's layout)."""
  C.check(C.lib.xse_tf32_split(x.data_ptr(), x.shape[0], x.shape[1],
                               x.stride(0), hi.data_ptr(), lo.data_ptr(),
                               stream_handle(stream)))


def linear_tf32x3(x_hi, x_lo, k_hi, k_lo, layer: DenseLayer, out, *,
                  stream=None):
  """out = act(x K + b) from split operands (xse_linear_forward_tf32x3)."""
  C.check(C.lib.xse_linear_forward_tf32x3(
      x_hi.data_ptr(), x_lo.data_ptr(), x_hi.shape[0], k_hi.shape[0],
      x_hi.stride(0), k_hi.data_ptr(), k_lo.data_ptr(), layer.bias.data_ptr(),
      k_hi.shape[1], layer.activation, out.data_ptr(), out.stride(0),
      stream_handle(stream)))
  return out


def linear(x, layer: DenseLayer, out, *, math=C.MATH_FP32, stream=None):
  """out = act(x[:, :in] K + b) through xse_linear_forward (x may be wider
  than the kernel's input: its row stride is passed)."""
  in_dim = layer.kernel.shape[0]
  rows = x.shape[0]
  C.check(C.lib.xse_linear_forward(
      x.data_ptr(), rows, in_dim, x.stride(0), layer.kernel.data_ptr(),
      layer.bias.data_ptr(), layer.kernel.shape[1], layer.activation, math,
      out.data_ptr(), out.stride(0), stream_handle(stream)))
  return out


class DenseTower:
  """Bottom MLP, dot interaction and top MLP on the device."""

  def __init__(self, num_dense=13, num_tables=26, dim=128, seed=0,
               bottom=BOTTOM_MLP, top=TOP_MLP, device="cuda",
               math=C.MATH_FP32):
    if bottom[-1] != dim:
      raise ValueError("The bottom MLP must end at the embedding dimension.")
    self.num_dense, self.num_tables, self.dim = num_dense, num_tables, dim
    self.width = interaction_width(num_tables, dim)
    # Interaction rows padded to a multiple of 4 floats: the interaction
    # writes zeros in the pad columns and the first top layer's kernel gets
    # zero rows there, so that GEMM runs with an aligned K (479 -> 480) and
    # the same result.
    self.width_stride = _round_up(self.width, 4)
    rng = np.random.default_rng(seed)
    self.host_bottom = init_dense_layers(num_dense, bottom, rng, False)
    self.host_top = init_dense_layers(self.width, top, rng, True)
    self.bottom = [self._upload(l, device) for l in self.host_bottom]
    self.top = [self._upload(l, device) for l in self.host_top]
    pad = self.width_stride - self.width
    if pad:
      k = self.top[0].kernel
      self.top[0].kernel = torch.cat(
          [k, torch.zeros((pad, k.shape[1]), dtype=k.dtype, device=k.device)])
    # Split-TF32 layers: every layer whose input width is a multiple of 4
    # except the 1-wide sigmoid head (own fp32 kernel); the 13-wide first
    # bottom layer stays on fp32 FMA (0.6 % of the tower's FLOPs).
    self._split = {}
    if math == MATH_TF32X3:
      for layer in self.bottom + self.top:
        k = layer.kernel
        if k.shape[0] % 4 == 0 and layer.activation != C.ACT_SIGMOID:
          hi, lo = torch.empty_like(k), torch.empty_like(k)
          tf32_split(k, hi, lo)
          self._split[id(layer)] = (hi, lo)
    self.device = device
    self.math = math
    self._buffers = {}

  @staticmethod
  def _upload(layer, device):
    kernel, bias, act = layer
    return DenseLayer(torch.from_numpy(kernel).to(device),
                      torch.from_numpy(bias).to(device), act)

  def _buffers_for(self, batch):
    bufs = self._buffers.get(batch)
    if bufs is None:
      f = dict(dtype=torch.float32, device=self.device)
      bufs = {
          "bottom": [torch.empty((batch, l.kernel.shape[1]), **f)
                     for l in self.bottom],
          "inter": torch.empty((batch, self.width_stride), **f),
          "top": [torch.empty((batch, l.kernel.shape[1]), **f)
                  for l in self.top],
          # split inputs of the widest layer, reused by every split layer
          "hi": torch.empty(batch * max(self.width_stride, 1024), **f),
          "lo": torch.empty(batch * max(self.width_stride, 1024), **f),
      }
      self._buffers[batch] = bufs
    return bufs

  def forward(self, dense, pooled, *, stream=None):
    """dense [B, num_dense] fp32, pooled [B, T, dim] fp32 (a sample's T rows
    contiguous) -> predictions [B] (a view of an internal buffer)."""
    x = self.bottom_forward(dense, stream=stream)
    inter = self.interaction_buffer(dense.shape[0])
    C.check(C.lib.xse_dot_interaction_strided(
        x.data_ptr(), x.stride(0), pooled.data_ptr(), pooled.stride(0),
        dense.shape[0], self.num_tables, self.dim, inter.data_ptr(),
        inter.stride(0), stream_handle(stream)))
    return self.top_forward(inter, stream=stream)

  def bottom_forward(self, dense, *, stream=None):
    """The bottom MLP: [B, num_dense] -> [B, dim] (an internal buffer)."""
    bufs = self._buffers_for(dense.shape[0])
    x = dense
    for layer, out in zip(self.bottom, bufs["bottom"]):
      x = self._layer(x, layer, out, bufs, stream)
    return x

  def interaction_buffer(self, batch):
    """The [B, width_stride] interaction rows the top MLP reads."""
    return self._buffers_for(batch)["inter"]

  def bottom_output(self, batch):
    """The bottom MLP's [B, dim] output buffer of the last forward."""
    return self._buffers_for(batch)["bottom"][-1]

  def interaction_rows(self, batch):
    """The [B, width_stride] interaction rows of the last forward."""
    return self.interaction_buffer(batch)

  def interaction_bytes_per_row(self):
    """Bytes of interaction output written per sample."""
    return self.width_stride * 4

  def split_launches(self, fused):
    """Operand-split kernels one forward launches: one per split layer,
    except the first top layer's when the fused interaction writes its
    operands."""
    return len(self._split) - (1 if fused and self.first_top_split() else 0)

  def first_top_split(self):
    """The split kernel of the first top layer, when it runs split-TF32 on
    the interaction rows as they are laid out (else None)."""
    return self._split.get(id(self.top[0]))

  def interaction_split_buffers(self, batch):
    """[B, width_stride] hi and lo views of the split scratch, where the
    fused interaction writes the first top layer's operands."""
    bufs = self._buffers_for(batch)
    n = batch * self.width_stride
    return (bufs["hi"][:n].view(batch, self.width_stride),
            bufs["lo"][:n].view(batch, self.width_stride))

  def top_forward_split(self, hi, lo, *, stream=None):
    """The top MLP from the first layer's split operands -> predictions."""
    bufs = self._buffers_for(hi.shape[0])
    layer = self.top[0]
    k_hi, k_lo = self._split[id(layer)]
    x = linear_tf32x3(hi, lo, k_hi, k_lo, layer, bufs["top"][0],
                      stream=stream)
    for layer, out in zip(self.top[1:], bufs["top"][1:]):
      x = self._layer(x, layer, out, bufs, stream)
    return x.view(-1)

  def top_forward(self, inter, *, stream=None):
    """The top MLP over interaction rows -> predictions [B]."""
    bufs = self._buffers_for(inter.shape[0])
    x = inter
    for layer, out in zip(self.top, bufs["top"]):
      x = self._layer(x, layer, out, bufs, stream)
    return x.view(-1)

  def _layer(self, x, layer, out, bufs, stream):
    split = self._split.get(id(layer))
    if split is not None and x.stride(0) != layer.kernel.shape[0]:
      split = None  # the split buffers are dense [rows, in]
    if split is None:
      math = C.MATH_FP32 if self.math == MATH_TF32X3 else self.math
      return linear(x, layer, out, math=math, stream=stream)
    rows, width = x.shape[0], layer.kernel.shape[0]
    hi = bufs["hi"][:rows * width].view(rows, width)
    lo = bufs["lo"][:rows * width].view(rows, width)
    tf32_split(x[:, :width], hi, lo, stream)
    return linear_tf32x3(hi, lo, split[0], split[1], layer, out, stream=stream)

  def reference_forward(self, dense, pooled):
    """The same forward in float64 torch on the host, for tests."""
    d = torch.as_tensor(np.asarray(dense), dtype=torch.float64)
    p = torch.as_tensor(np.asarray(pooled), dtype=torch.float64)
    x = d
    for kernel, bias, _ in self.host_bottom:
      x = torch.relu(x @ torch.from_numpy(kernel).double() +
                     torch.from_numpy(bias).double())
    z = torch.cat([x[:, None, :], p], dim=1)
    gram = z @ z.transpose(1, 2)
    rows = self.num_tables + 1
    iu = torch.triu_indices(rows, rows, offset=1)
    x = torch.cat([x, gram[:, iu[0], iu[1]]], dim=1)
    for k, (kernel, bias, act) in enumerate(self.host_top):
      x = x @ torch.from_numpy(kernel).double() + torch.from_numpy(bias).double()
      x = torch.sigmoid(x) if act == C.ACT_SIGMOID else torch.relu(x)
    return x.view(-1).numpy()


class DLRM:
  """Embedding lookups of the sparse features plus the dense tower."""

  def __init__(self, engine: EmbeddingEngine, feature_names: Sequence[str],
               dim=128, num_dense=13, seed=0, device="cuda",
               math=C.MATH_FP32, fused_interaction=True):
    self.engine = engine
    # Pooling and the dot interaction in one engine call
    # (execute_interaction): the pooled rows stay on chip.
    self.fused_interaction = fused_interaction
    self.features = list(feature_names)
    self.dim = dim
    self.tower = DenseTower(num_dense, len(self.features), dim, seed,
                            device=device, math=math)
    self.device = device
    self._pooled = {}

  def pooled_buffer(self, batch):
    buf = self._pooled.get(batch)
    if buf is None:
      buf = torch.empty((batch, len(self.features), self.dim),
                        dtype=torch.float32, device=self.device)
      self._pooled[batch] = buf
    return buf

  def requests(self, ids: List[torch.Tensor], offsets: List[torch.Tensor],
               weights: Optional[List[Optional[torch.Tensor]]] = None):
    """Bag requests writing each feature into its slot of the pooled
    [B, T, dim] buffer (strided outputs, one group)."""
    batch = offsets[0].numel() - 1
    pooled = self.pooled_buffer(batch)
    t = len(self.features)
    reqs = []
    for k, name in enumerate(self.features):
      w = None if weights is None else weights[k]
      reqs.append(BagRequest(name, ids[k], offsets[k], pooled[:, k, :], w,
                             output_stride=t * self.dim))
    return reqs, pooled

  def forward(self, dense, ids=None, offsets=None, weights=None, *,
              requests=None, status: Optional[Status] = None, stream=None):
    """Predictions [B] for dense features [B, num_dense] and per-feature CSR
    ids/offsets (or prebuilt `requests` from requests())."""
    if requests is None:
      requests, pooled = self.requests(ids, offsets, weights)
    else:
      pooled = self.pooled_buffer(dense.shape[0])
    # Fused checks: the pooled rows are internal to the forward, so a
    # failing group need not leave them untouched (the error is still
    # raised, or reported by status.wait()); no separate validation pass.
    if self.fused_interaction:
      x = self.tower.bottom_forward(dense, stream=stream)
      batch = dense.shape[0]
      if self.tower.first_top_split() is not None:
        # The interaction kernel writes the first top layer's split-TF32
        # operands: no split pass over the interaction rows.
        hi, lo = self.tower.interaction_split_buffers(batch)
        self.engine.execute_interaction(requests, x, hi, stream=stream,
                                        status=status, fused=True, out_lo=lo)
        return self.tower.top_forward_split(hi, lo, stream=stream)
      inter = self.tower.interaction_buffer(batch)
      self.engine.execute_interaction(requests, x, inter, stream=stream,
                                      status=status, fused=True)
      return self.tower.top_forward(inter, stream=stream)
    self.engine.execute_batch(requests, stream=stream, status=status,
                              fused=True)
    return self.tower.forward(dense, pooled, stream=stream)
