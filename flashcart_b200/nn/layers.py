"""Layers of the FlashCart potential on the B200 operators.

Same classes, constructor arguments, parameter/buffer names, persistence and
parameter-creation order as the reference ``nn/layers.py`` (so reference
checkpoints load unchanged and a seeded construction draws the same random
weights); every equivariant operation (tensor products, linear maps) goes through
:mod:`flashcart_b200.o3`, i.e. the sm_100a kernels, and so do the dense layers of the
radial / readout MLPs and gates (as one-rank linear maps on the tensor cores).
"""

from typing import Iterator, List, Optional

import torch
import torch.nn as nn
import torch.nn.functional as F

from flashcart_b200 import o3, ops


def iter_child_special_parameters(module: nn.Module, method_name: str) -> Iterator[nn.Parameter]:
    """Each parameter reported by the ``method_name`` hook of any nested child (not the
    module itself), once (reference ``utils/parameter_groups.py:6-30``). The hooks route
    parameters away from Muon / weight decay in the optimizer factory."""
    seen = set()
    for child in module.modules():
        if child is module:
            continue
        method = getattr(child, method_name, None)
        if method is None:
            continue
        for p in method():
            if id(p) not in seen:
                seen.add(id(p))
                yield p


class _NoSpecialParameters:
    def non_decayable_parameters(self) -> Iterator[nn.Parameter]:
        return iter(())

    def non_muon_parameters(self) -> Iterator[nn.Parameter]:
        return iter(())


class _ChildSpecialParameters:
    def non_decayable_parameters(self) -> Iterator[nn.Parameter]:
        yield from iter_child_special_parameters(self, "non_decayable_parameters")

    def non_muon_parameters(self) -> Iterator[nn.Parameter]:
        yield from iter_child_special_parameters(self, "non_muon_parameters")


class RescaledSiLULayer(_NoSpecialParameters, nn.Module):
    """scale * silu(x); default scale 1/sqrt(E[silu(z)^2]), z ~ N(0,1) (reference ``nn/layers.py:12-44``)."""

    def __init__(self, scale: Optional[float] = None):
        super().__init__()
        self.register_buffer("scale", torch.tensor(1.6765324703310907 if scale is None else scale,
                                                   dtype=torch.get_default_dtype()), persistent=False)

    def forward(self, x):
        return self.scale * F.silu(x)


class RescaledSigmoidLayer(_NoSpecialParameters, nn.Module):
    """scale * sigmoid(x); default scale 1/sqrt(E[sigmoid(z)^2]) (reference ``nn/layers.py:47-79``)."""

    def __init__(self, scale: Optional[float] = None):
        super().__init__()
        self.register_buffer("scale", torch.tensor(1.8462285453386054 if scale is None else scale,
                                                   dtype=torch.get_default_dtype()), persistent=False)

    def forward(self, x):
        return self.scale * torch.sigmoid(x)


class LinearLayer(nn.Module):
    """y = x (scale W)^T + b with N(0,1) W and scale 1/sqrt(in) (reference ``nn/layers.py:82-140``).

    Evaluated by the tensor-core kernel of ``flashcart::linear_fwd`` (one rank, one
    component: a plain row-major GEMM), fp32 as 3xTF32, so the radial and readout MLPs
    (1.5 M edge rows at the benchmark size) run on tcgen05 instead of fp32 SIMT.
    """

    def __init__(self, in_features: int, out_features: int, bias: bool = False,
                 weight_scale: Optional[float] = None):
        super().__init__()
        self.in_features = in_features
        self.out_features = out_features
        s = float(in_features) ** -0.5 if weight_scale is None else float(weight_scale)
        self.register_buffer("scale", torch.tensor(s, dtype=torch.get_default_dtype()), persistent=False)
        self.weight = nn.Parameter(torch.randn(out_features, in_features))
        if bias:
            self.bias = nn.Parameter(torch.zeros(out_features))
        else:
            self.register_parameter("bias", None)
        self._meta = torch.zeros(1, 6, dtype=torch.int64)
        self._lists = ([0], [0], [0], [1], [in_features], [out_features])

    def silu_input_fusable(self, x) -> bool:
        """The SiLU of the input can be applied inside this layer's GEMM (first derivative
        only, frozen weights, float32 on the GPU, at most 64 inputs: the input gradient's
        SiLU' epilogue exists for 64-column tiles; row widths in 16-byte units for TMA)."""
        return (ops.first_order_only_active() and x.is_cuda and x.dtype == torch.float32
                and self.weight.dtype == torch.float32 and not self.weight.requires_grad
                and self.in_features <= 64 and self.in_features % 4 == 0 and self.out_features % 4 == 0)

    def forward(self, x, input_scale: Optional[torch.Tensor] = None, silu_input: bool = False):
        """``input_scale`` (optional 0-d tensor) multiplies the input; the map is linear, so it
        is applied to the layer's scale instead of to every element of ``x``. ``silu_input``
        makes the layer act on silu(x) (inside its GEMM when :meth:`silu_input_fusable`)."""
        lead = x.shape[:-1]
        x2 = x.reshape(-1, self.in_features)
        use_fp64, precision = o3.utils.get_linear_triton_kernel_options(x.dtype)
        w = self.weight if self.weight.dtype == x.dtype else self.weight.to(x.dtype)
        scale = self.scale.reshape(1) if input_scale is None else self.scale.reshape(1) * input_scale
        if silu_input and self.silu_input_fusable(x2):
            y = torch.ops.flashcart.linear_silu_fwd(x2, [w], self.out_features, precision, self._lists[0],
                                                    self._lists[1], self._lists[3], self._lists[4], self._lists[5],
                                                    scale)
            if self.bias is not None:
                y = y + self.bias
            return y.reshape(*lead, self.out_features)
        if silu_input:
            x2 = F.silu(x2)
        y = torch.ops.flashcart.linear_fwd(x2, [w], self._meta, self.out_features, use_fp64, precision,
                                           *self._lists, scale)
        if self.bias is not None:
            y = y + self.bias
        return y.reshape(*lead, self.out_features)


def _linear_non_decayable(self) -> Iterator[nn.Parameter]:
    if self.bias is not None:
        yield self.bias


LinearLayer.non_decayable_parameters = _linear_non_decayable
LinearLayer.non_muon_parameters = _linear_non_decayable


class _MLP(nn.Sequential):
    """Linear / rescaled-SiLU stack (the reference's ``nn.Sequential``, same state_dict keys).
    The constant of each rescaled SiLU is handed to the next linear layer's scale instead of
    being multiplied into the activations (one pass over the edge rows less per layer), and
    the SiLU itself is applied by that layer: inside its GEMM in first-order evaluation with
    frozen weights (no activation tensor is written; SiLU' is applied in the input
    gradient's epilogue), else as a separate elementwise pass."""

    def forward(self, x):
        mods = list(self)
        pending = None
        for k, m in enumerate(mods):
            if isinstance(m, RescaledSiLULayer) and k + 1 < len(mods) and isinstance(mods[k + 1], LinearLayer):
                # the next linear layer applies the SiLU to its input (inside its GEMM where
                # possible) and takes the rescale into its weight scale
                pending = m.scale
            elif isinstance(m, LinearLayer):
                x = m(x, input_scale=pending, silu_input=pending is not None)
                pending = None
            else:
                x = m(x)
        return x


def _mlp(widths: List[int]) -> nn.Sequential:
    layers = []
    for a, b in zip(widths[:-1], widths[1:]):
        layers.append(LinearLayer(a, b))
        layers.append(RescaledSiLULayer())
    return _MLP(*layers[:-1])


class RMSLayerNorm(nn.Module):
    """Normalise Cartesian features by an invariant mean square (reference ``nn/layers.py:413-540``).

    The invariant squared norm of every rank comes from a symmetric scalar tensor
    product (shared unit weights), weighted 1/((2l+1)(l_max+1)) and averaged over
    channels; per-rank gains (and an l=0 bias with centering) follow.
    """

    def non_decayable_parameters(self) -> Iterator[nn.Parameter]:
        yield from self.parameters()

    def non_muon_parameters(self) -> Iterator[nn.Parameter]:
        yield from self.parameters()

    def __init__(self, l_max: int, n_features: int, eps: float = 1.0e-12, affine: bool = True,
                 centering: bool = False, use_triton: bool = False):
        super().__init__()
        self.l_max = l_max
        self.n_features = n_features
        self.eps = eps
        self.affine = affine
        self.centering = centering
        self.slices = o3.utils.get_irreps_slices(l_max, n_features)
        self.shapes = o3.utils.get_irreps_shapes(l_max, n_features)
        self.block_dims = [a * b for a, b in self.shapes]
        self.dim = sum(self.block_dims)
        self.tp = o3.TensorProduct(l_max, l_max, 0, n_features, n_features, use_triton=use_triton,
                                   symmetric_product=True, shared_weights=True, reduce_paths=False)
        _, n_paths = o3.utils.count_output_paths(l_max, l_max, 0, symmetric_product=True)
        self.register_buffer("dummy_tp_weights", torch.ones(n_paths * n_features), persistent=False)
        self.register_buffer("l_weights", torch.tensor([1.0 / ((2 * l + 1) * (l_max + 1)) for l in range(l_max + 1)],
                                                       dtype=torch.float64), persistent=False)
        if affine:
            self.weights = nn.ParameterList([nn.Parameter(torch.ones(n_features)) for _ in range(l_max + 1)])
            reps = torch.tensor([2 * l + 1 for l in range(l_max + 1)])
            self.register_buffer("l_expand_index", torch.arange(l_max + 1).repeat_interleave(reps),
                                 persistent=False)
            if centering:
                self.bias = nn.Parameter(torch.zeros(n_features))
            else:
                self.register_parameter("bias", None)
        else:
            self.weights = nn.ParameterList()
            self.register_parameter("bias", None)

    def _fused_ok(self, node_feats: torch.Tensor) -> bool:
        """The fused kernel pair (one pass forward, one backward) replaces the composition
        when the graph is differentiated at most once, without centering, with constant
        gains (parameters frozen, as in force / stress evaluation)."""
        return (ops.first_order_only_active() and node_feats.is_cuda and node_feats.dim() == 2
                and not self.centering and node_feats.dtype in (torch.float32, torch.float64)
                and not any(w.requires_grad for w in self.weights))

    def forward(self, node_feats: torch.Tensor) -> torch.Tensor:
        if node_feats.shape[-1] != self.dim:
            raise RuntimeError(f"Incorrect last dimension for node_feats. Expected {self.dim}, "
                               f"got {node_feats.shape[-1]}.")
        if self._fused_ok(node_feats):
            gains = (torch.stack(tuple(self.weights)) if self.affine else
                     node_feats.new_ones((self.l_max + 1, self.n_features)))
            return ops.rms_norm(node_feats, gains, self.l_weights, self.l_max, self.n_features, self.eps)
        n = node_feats.shape[0]
        feats = node_feats
        if self.centering:
            l0 = node_feats[:, :self.n_features]
            feats = torch.cat([l0 - l0.mean(dim=-1, keepdim=True), node_feats[:, self.n_features:]], dim=-1)
        inv = self.tp(feats, feats, self.dummy_tp_weights.to(feats.dtype)).view(n, self.l_max + 1, self.n_features)
        mean_sq = (inv * self.l_weights.to(inv.dtype).view(1, -1, 1)).sum(dim=1).mean(dim=-1, keepdim=True)
        scaled = feats * torch.pow(mean_sq + self.eps, -0.5)
        if not self.affine:
            return scaled
        gains = torch.stack(tuple(self.weights)).index_select(0, self.l_expand_index).view(1, -1)
        out = scaled * gains
        if self.bias is not None:
            out = torch.cat([out[:, :self.n_features] + self.bias, out[:, self.n_features:]], dim=-1)
        return out


class InteractionLayer(nn.Module):
    """Tensor-product convolution with radial-MLP path weights (reference ``nn/layers.py:184-410``).

    node feats -> linear_first -> conv TP with edge attributes, weights =
    radial_mlp(basis * envelope) -> / sqrt(avg_neighbors) -> linear_second
    (+ skip projection) (-> RMS layer norm).
    """

    def non_decayable_parameters(self) -> Iterator[nn.Parameter]:
        yield from iter_child_special_parameters(self, "non_decayable_parameters")

    def non_muon_parameters(self) -> Iterator[nn.Parameter]:
        yield from iter_child_special_parameters(self, "non_muon_parameters")
        if self.emb_i is not None:
            yield from self.emb_i.parameters()
            yield from self.emb_j.parameters()

    def __init__(self, in1_l_max: int, in2_l_max: int, out_l_max: int, in1_features: int, out_features: int,
                 n_radial: int, hidden_radial: Optional[List[int]] = None, n_elements: Optional[int] = None,
                 element_features: Optional[int] = None, avg_neighbors: float = 1.0, use_sc: bool = False,
                 use_layer_norm: bool = False, use_triton: bool = False, recompute_radial: bool = False):
        super().__init__()
        self.in1_l_max, self.in2_l_max, self.out_l_max = in1_l_max, in2_l_max, out_l_max
        self.in1_features, self.out_features = in1_features, out_features
        self.n_radial = n_radial
        self.hidden_radial = [64, 64] if hidden_radial is None else list(hidden_radial)
        self.use_sc = use_sc
        self.use_layer_norm = use_layer_norm
        self.recompute_radial = recompute_radial
        if avg_neighbors <= 0.0:
            raise ValueError(f"avg_neighbors must be positive. Provided: {avg_neighbors}.")
        self.register_buffer("sqrt_avg_neighbors",
                             torch.tensor(float(avg_neighbors) ** 0.5, dtype=torch.get_default_dtype()))
        self.out_dim = sum((2 * l + 1) * out_features for l in range(out_l_max + 1))
        out_paths, n_total_paths = o3.utils.count_output_paths(in1_l_max, in2_l_max, out_l_max)
        if n_elements is not None and element_features is None:
            raise ValueError("element_features must be provided when n_elements is set.")
        self.element_features = element_features
        radial_in = n_radial + 2 * element_features if n_elements is not None else n_radial
        self.radial_mlp = _mlp([radial_in] + self.hidden_radial + [n_total_paths * in1_features])
        self.tp = o3.TensorProduct(in1_l_max, in2_l_max, out_l_max, in1_features, 1, use_triton=use_triton,
                                   reduce_paths=False)
        self.linear_first = o3.LinearLayer(in1_l_max, in1_l_max, in1_features, in1_features, use_triton=use_triton)
        self.linear_second = o3.LinearLayer(out_l_max, out_l_max, in1_features, out_features, in_paths=out_paths,
                                            use_triton=use_triton)
        if use_sc:
            self.skip_projection = (LinearLayer(in1_features, out_features) if in1_l_max == 0 else
                                    o3.LinearLayer(in1_l_max, out_l_max, in1_features, out_features,
                                                   use_triton=use_triton))
        else:
            self.skip_projection = None
        self.layer_norm = (RMSLayerNorm(out_l_max, out_features, eps=1.0e-6, use_triton=use_triton)
                           if use_layer_norm else None)
        if n_elements is not None:
            self.emb_i = nn.Embedding(n_elements, element_features)
            self.emb_j = nn.Embedding(n_elements, element_features)
            nn.init.uniform_(self.emb_i.weight, a=-0.001, b=0.001)
            nn.init.uniform_(self.emb_j.weight, a=-0.001, b=0.001)
        else:
            self.emb_i = None
            self.emb_j = None

    def forward(self, node_feats, edge_attrs, edge_feats, edge_index, envelope, atom_types=None, out_nodes=None):
        idx_i, idx_j = edge_index[0], edge_index[1]
        residual = node_feats if out_nodes is None else node_feats[:out_nodes]
        if self.emb_i is not None:
            if atom_types is None:
                raise ValueError(f"atom_types required when n_elements is set. Provided: {atom_types}.")
            mlp_in = torch.cat([edge_feats, self.emb_i(atom_types)[idx_i], self.emb_j(atom_types)[idx_j]], dim=-1)
            mlp_in = mlp_in * envelope.unsqueeze(-1)
        else:
            # envelope None: edge_feats already carries the envelope (fused edge geometry)
            mlp_in = edge_feats if envelope is None else edge_feats * envelope.unsqueeze(-1)
        node_feats = self.linear_first(node_feats)
        weights = self.radial_mlp(mlp_in)
        aggregated = self.tp(node_feats, edge_attrs, weights, idx_i, idx_j)
        if out_nodes is not None:
            aggregated = aggregated[:out_nodes]
        # aggregated / sqrt(avg_neighbors), folded into the scales of the linear map
        if self.skip_projection is not None and self.in1_l_max != 0:
            # the skip projection is added in linear_second's epilogue where that is possible
            out = self.linear_second(aggregated, input_scale=1.0 / self.sqrt_avg_neighbors,
                                     residual=self.skip_projection(residual))
        else:
            out = self.linear_second(aggregated, input_scale=1.0 / self.sqrt_avg_neighbors)
        if self.skip_projection is not None and self.in1_l_max == 0:
            # the skip reaches the l = 0 block only: added in place into the fresh output of
            # linear_second (whose backward does not read it) instead of concatenating a new
            # row (a copy of every rank block, and in the backward a zero-filled row per slice
            # plus their sum)
            out[:, :self.out_features].add_(self.skip_projection(residual))
        if self.layer_norm is not None:
            out = self.layer_norm(out)
        return out

    def set_avg_neighbors(self, avg_neighbors: float) -> None:
        if avg_neighbors <= 0.0:
            raise ValueError(f"avg_neighbors must be positive. Provided: {avg_neighbors}.")
        self.sqrt_avg_neighbors.fill_(float(avg_neighbors) ** 0.5)


class EquivariantGatedLayer(_ChildSpecialParameters, nn.Module):
    """Gated residual update, identity at initialisation (reference ``nn/layers.py:543-648``)."""

    def __init__(self, l_max: int, in_features: int, hidden_features: Optional[int] = None,
                 gate_activation: str = "silu", gate_bias: bool = True, use_triton: bool = False):
        super().__init__()
        if gate_activation not in ("silu", "sigmoid"):
            raise ValueError(f"gate_activation must be 'silu' or 'sigmoid'. Provided: {gate_activation!r}.")
        self.l_max = l_max
        self.in_features = in_features
        self.gate_activation_name = gate_activation
        self.gate_bias = gate_bias
        self.hidden_features = in_features if hidden_features is None else hidden_features
        if self.hidden_features <= 0:
            raise ValueError(f"hidden_features must be positive. Provided: {self.hidden_features}.")
        self.in_dim = sum((2 * l + 1) * in_features for l in range(l_max + 1))
        self.hidden_dim = sum((2 * l + 1) * self.hidden_features for l in range(l_max + 1))
        self.hidden_slices = o3.utils.get_irreps_slices(l_max, self.hidden_features)
        self.value_linear = o3.LinearLayer(l_max, l_max, in_features, self.hidden_features, use_triton=use_triton)
        self.gate_linear = LinearLayer(in_features, (l_max + 1) * self.hidden_features, bias=gate_bias)
        self.gate_activation = RescaledSiLULayer() if gate_activation == "silu" else RescaledSigmoidLayer()
        self.output_linear = o3.LinearLayer(l_max, l_max, self.hidden_features, in_features, use_triton=use_triton)
        for w in self.output_linear.weight:
            nn.init.zeros_(w)

    def _fused_ok(self, node_feats) -> bool:
        """One autograd node for the whole layer (first-order evaluation, frozen float32
        weights, the residual-epilogue layout for both equivariant maps)."""
        if not (ops.first_order_only_active() and node_feats.is_cuda and node_feats.dtype == torch.float32
                and node_feats.is_contiguous() and node_feats.data_ptr() % 16 == 0
                and not any(p.requires_grad for p in self.parameters())):
            return False
        for lin in (self.value_linear, self.output_linear):
            in_offs, out_offs, _, m, fi, fo = lin.meta_lists
            if not ops.linear_residual_layout_ok(lin.in_dim, lin.out_dim, m, fi, fo, in_offs, out_offs):
                return False
        return self.gate_linear.in_features % 4 == 0 and self.gate_linear.out_features % 4 == 0

    def forward(self, node_feats):
        if node_feats.shape[-1] != self.in_dim:
            raise RuntimeError(f"Incorrect last dimension for node_feats. Expected {self.in_dim}, "
                               f"got {node_feats.shape[-1]}.")
        if self._fused_ok(node_feats):
            return _GatedResidualFirstOrder.apply(node_feats, self)
        n = node_feats.shape[0]
        values = self.value_linear(node_feats)
        gates = self.gate_activation(self.gate_linear(node_feats[:, :self.in_features]))
        gates = gates.view(n, self.l_max + 1, self.hidden_features)
        if ops.first_order_only_active() and values.is_cuda and values.dtype in (torch.float32, torch.float64):
            # one fused pass over the rank blocks (first derivative only)
            gated = ops.gate_fwd(values, gates, self.l_max, self.hidden_features)
            # the residual is added in the output map's epilogue where that is possible
            return self.output_linear(gated, residual=node_feats)
        parts = []
        for l, (a, b) in enumerate(self.hidden_slices):
            parts.append((values[:, a:b].view(n, 2 * l + 1, self.hidden_features) * gates[:, l].unsqueeze(1))
                         .flatten(1))
        return node_feats + self.output_linear(torch.cat(parts, dim=-1))


class _GatedResidualFirstOrder(torch.autograd.Function):
    """``EquivariantGatedLayer`` as one autograd node for first-order evaluation with frozen
    weights. The input feeds three consumers (the value map, the gate map through its l = 0
    block, and the residual); composed, their gradients are summed by separate passes over
    the rows (and the l = 0 slice's gradient is first written into a zero-filled row). Here
    the value map's input gradient is computed with the incoming gradient as its residual
    (one GEMM epilogue) and the gate map's gradient is added into the l = 0 block."""

    @staticmethod
    def forward(ctx, node_feats, layer):
        n = node_feats.shape[0]
        values = layer.value_linear(node_feats)
        gpre = layer.gate_linear(node_feats[:, :layer.in_features])
        gates = layer.gate_activation(gpre).view(n, layer.l_max + 1, layer.hidden_features)
        gated = ops.gate_fwd(values, gates, layer.l_max, layer.hidden_features)
        out = layer.output_linear(gated, residual=node_feats)
        ctx.save_for_backward(values, gates, gpre)
        ctx.layer = layer
        return out

    @staticmethod
    def backward(ctx, g):
        if torch.is_grad_enabled():
            raise RuntimeError("EquivariantGatedLayer was evaluated inside first_order_only(); its backward cannot "
                               "build a graph for a second derivative")
        values, gates, gpre = ctx.saved_tensors
        layer = ctx.layer
        g = g.contiguous()
        if g.data_ptr() % 16:  # the epilogue reads the residual as 16-byte vectors
            g = g.clone()
        _, precision = o3.utils.get_linear_triton_kernel_options(g.dtype)
        out_map, value_map, gate_map = layer.output_linear, layer.value_linear, layer.gate_linear
        g_gated = ops._linear_input_grad(g, out_map.in_dim, list(out_map.weight), out_map.meta_lists, precision,
                                         out_map.scale)
        g_values, g_gates = ops.gate_bwd(g_gated, values, gates, layer.l_max, layer.hidden_features)
        with torch.enable_grad():
            gp = gpre.detach().requires_grad_(True)
            (g_gpre,) = torch.autograd.grad(layer.gate_activation(gp), gp, g_gates.reshape(gpre.shape))
        # value map's input gradient + the residual's gradient, in one epilogue
        g_x = ops._linear_residual_impl(g_values.contiguous(), list(value_map.weight), value_map.in_dim,
                                        value_map.meta_lists, precision, value_map.scale, g, True)
        g_x0 = ops._linear_input_grad(g_gpre.contiguous(), gate_map.in_features, [gate_map.weight],
                                      gate_map._lists, precision, gate_map.scale.reshape(1))
        g_x[:, :layer.in_features] += g_x0
        return g_x, None


class IrrepsSelector(_NoSpecialParameters, nn.Module):
    """Keep the leading rank blocks up to out_l_max (reference ``nn/layers.py:651-698``)."""

    def __init__(self, in_l_max: int, out_l_max: int, in_features: int, in_paths: Optional[List[int]] = None):
        super().__init__()
        if out_l_max > in_l_max:
            raise ValueError("out_l_max must be less than or equal to in_l_max. "
                             f"Provided: out_l_max={out_l_max}, in_l_max={in_l_max}.")
        in_paths = [1] * (in_l_max + 1) if in_paths is None else list(in_paths)
        self.stop = o3.utils.get_irreps_slices(in_l_max, in_features, in_paths)[out_l_max][1]
        self.in_dim = sum((2 * l + 1) * in_features * in_paths[l] for l in range(in_l_max + 1))

    def forward(self, x):
        if x.shape[-1] != self.in_dim:
            raise RuntimeError(f"Incorrect last dimension for x. Expected {self.in_dim}, got {x.shape[-1]}.")
        return x[:, :self.stop]


class ProductPathWeights(nn.Module):
    """Per-path multiplicative weights 1 + delta (reference ``nn/layers.py:701-765``)."""

    def non_decayable_parameters(self) -> Iterator[nn.Parameter]:
        return iter(())

    def non_muon_parameters(self) -> Iterator[nn.Parameter]:
        if not self.learnable:
            return
        if self.element_dependent:
            yield from self.delta.parameters()
        else:
            yield self.delta

    def __init__(self, n_weights: int, n_elements: Optional[int] = None, learnable: bool = False):
        super().__init__()
        if n_elements is not None and not learnable:
            raise ValueError("Element-dependent path weights must be learnable. "
                             "Provided: learnable=False with n_elements set.")
        self.learnable = learnable
        self.element_dependent = False
        if not learnable:
            self.register_buffer("delta", torch.zeros(n_weights), persistent=False)
        elif n_elements is None:
            self.delta = nn.Parameter(torch.zeros(n_weights))
        else:
            self.element_dependent = True
            self.delta = nn.Embedding(n_elements, n_weights)
            nn.init.zeros_(self.delta.weight)

    def forward(self, atom_types=None):
        if self.element_dependent:
            if atom_types is None:
                raise ValueError("atom_types required when n_elements is set.")
            return 1.0 + self.delta(atom_types)
        return 1.0 + self.delta


class ProductLayer(_ChildSpecialParameters, nn.Module):
    """Repeated node-local products up to the correlation order (reference ``nn/layers.py:768-1018``)."""

    def __init__(self, in_l_max: int, out_l_max: int, in_features: int, n_elements: Optional[int] = None,
                 correlation: int = 2, path_reduced: bool = False, use_sc: bool = False,
                 use_layer_norm: bool = False, use_triton: bool = False):
        super().__init__()
        if correlation < 2:
            raise ValueError("ProductLayer requires correlation >= 2. "
                             "Use FlashCartPotential(correlation=1) for an interaction-only model.")
        self.in_l_max, self.out_l_max, self.in_features = in_l_max, out_l_max, in_features
        self.correlation = correlation
        self.path_reduced = path_reduced
        self.learnable_path_weights = path_reduced or n_elements is not None
        self.use_sc = use_sc
        self.use_layer_norm = use_layer_norm
        self.in_dim = sum((2 * l + 1) * in_features for l in range(in_l_max + 1))
        self.out_dim = sum((2 * l + 1) * in_features for l in range(out_l_max + 1))
        self.skip_projection = (o3.LinearLayer(in_l_max, out_l_max, in_features, in_features, use_triton=use_triton)
                                if use_sc else None)
        self.layer_norm = (RMSLayerNorm(out_l_max, in_features, eps=1.0e-6, use_triton=use_triton)
                           if use_layer_norm else None)
        if path_reduced:
            self.final_linear = o3.LinearLayer(out_l_max, out_l_max, in_features, in_features, use_triton=use_triton)
        self.tensor_products = nn.ModuleList()
        self.path_weights = nn.ModuleList()
        self.irreps_selectors = nn.ModuleList()
        self.product_linears = nn.ModuleList()
        self.path_norm_names: List[Optional[str]] = []
        for step in range(correlation):
            step_out = out_l_max if step == correlation - 1 else in_l_max
            in2_l_max, in2_features = (0, 1) if step == 0 else (in_l_max, in_features)
            out_paths, n_total = o3.utils.count_output_paths(in_l_max, in2_l_max, step_out, symmetric_product=False)
            self.path_weights.append(ProductPathWeights(n_total * in_features, n_elements=n_elements,
                                                        learnable=self.learnable_path_weights))
            if path_reduced:
                norm = torch.cat([torch.full(((2 * l + 1) * in_features,), out_paths[l] ** -0.5)
                                  for l in range(step_out + 1)])
                if torch.all(norm == 1.0):
                    self.path_norm_names.append(None)
                else:
                    name = f"path_norm_{step}"
                    self.register_buffer(name, norm)
                    self.path_norm_names.append(name)
            else:
                self.product_linears.append(o3.LinearLayer(step_out, step_out if step < correlation - 1 else out_l_max,
                                                           in_features, in_features, in_paths=out_paths,
                                                           use_triton=use_triton))
            self.irreps_selectors.append(nn.Identity() if step_out == out_l_max else
                                         IrrepsSelector(step_out, out_l_max, in_features))
            if step > 0:
                self.tensor_products.append(o3.TensorProduct(in_l_max, in2_l_max, step_out, in_features, in2_features,
                                                             use_triton=use_triton, reduce_paths=path_reduced,
                                                             symmetric_product=False,
                                                             shared_weights=n_elements is None))
        if self.learnable_path_weights:
            self.register_buffer("step0_weight_index", torch.cat(
                [torch.arange(l * in_features, (l + 1) * in_features).repeat(2 * l + 1) for l in range(in_l_max + 1)]),
                persistent=False)
        else:
            self.step0_weight_index = None

    def _selected_comps(self) -> Optional[int]:
        """Leading components of a step's output that enter the sum (all when its selector is
        the identity), or None when the steps select differently."""
        comps = set()
        d = (self.in_l_max + 1) ** 2
        for sel in self.irreps_selectors:
            if isinstance(sel, nn.Identity):
                continue
            if sel.stop % self.in_features:
                return None
            comps.add(sel.stop // self.in_features)
        return d if not comps else (comps.pop() if len(comps) == 1 else None)

    def _single_node_ok(self, node_feats) -> bool:
        """One autograd node for the whole layer: first-order evaluation, frozen float32
        weights shared by all atoms, no step-0 weighting, paths kept, the products on the
        dense channel-pair kernels (64 or 128 channels)."""
        if not (ops.first_order_only_active() and node_feats.is_cuda and node_feats.dtype == torch.float32
                and node_feats.is_contiguous() and node_feats.data_ptr() % 16 == 0 and not self.path_reduced
                and self.skip_projection is not None and self.step0_weight_index is None
                and self.in_features in (64, 128) and self._selected_comps() is not None
                and not any(p.requires_grad for p in self.parameters())):
            return False
        return all(tp.in1_features == tp.in2_features and not tp.reduce_paths for tp in self.tensor_products)

    def forward(self, node_feats, atom_types=None):
        if self._single_node_ok(node_feats):
            ws = [self.path_weights[step](atom_types).to(node_feats.dtype).contiguous()
                  for step in range(1, self.correlation)]
            out = _ProductSumFirstOrder.apply(node_feats, self, *ws)
            return self.layer_norm(out) if self.layer_norm is not None else out
        if (not self.path_reduced and self.skip_projection is not None
                and all(isinstance(s, nn.Identity) for s in self.irreps_selectors)):
            return self._forward_summed_in_maps(node_feats, atom_types)
        out = None  # sum of the selected products (the reference starts from zeros; 0 + x == x)
        prod = node_feats
        for step in range(self.correlation):
            if step == 0:
                if self.step0_weight_index is not None:
                    w = self.path_weights[0](atom_types)
                    prod = node_feats * w[..., self.step0_weight_index]
                else:
                    prod = node_feats
            else:
                w = self.path_weights[step](atom_types).to(node_feats.dtype)
                prod = self.tensor_products[step - 1](prod, node_feats, w)
            if self.path_reduced:
                name = self.path_norm_names[step]
                if name is not None:
                    prod = prod * getattr(self, name)
            else:
                prod = self.product_linears[step](prod)
            sel = self.irreps_selectors[step](prod)
            out = sel if out is None else out + sel
        if self.path_reduced:
            out = self.final_linear(out)
        if self.skip_projection is not None:
            out = out + self.skip_projection(node_feats)
        if self.layer_norm is not None:
            out = self.layer_norm(out)
        return out


    def _forward_summed_in_maps(self, node_feats, atom_types=None):
        """The same sum (every step's product, all ranks kept, plus the skip projection) with
        the additions moved into the maps that produce their terms: the skip projection adds
        the first product and the last product map adds the rest (in their GEMM epilogues
        where ``ops.linear_residual_fusable`` allows), so only the middle products are
        summed separately."""
        prods, prod = [], node_feats
        for step in range(self.correlation):
            if step == 0:
                if self.step0_weight_index is not None:
                    w = self.path_weights[0](atom_types)
                    prod = node_feats * w[..., self.step0_weight_index]
            else:
                w = self.path_weights[step](atom_types).to(node_feats.dtype)
                prod = self.tensor_products[step - 1](prod, node_feats, w)
            if step < self.correlation - 1:
                prod = self.product_linears[step](prod)
                prods.append(prod)
        acc = self.skip_projection(node_feats, residual=prods[0])
        for p in prods[1:]:
            acc = acc + p
        out = self.product_linears[self.correlation - 1](prod, residual=acc)
        if self.layer_norm is not None:
            out = self.layer_norm(out)
        return out


class _ProductSumFirstOrder(torch.autograd.Function):
    """``ProductLayer`` (before its layer norm) as one autograd node for first-order
    evaluation with frozen weights. Composed, every input of the layer's sum has several
    consumers: the node features feed the first map, every product and the skip projection;
    each intermediate product feeds the next product and the sum (through a slice when the
    layer keeps only the low ranks). Their gradients are then summed by separate passes
    over the rows, after zero-filled rows for the slices. Here the backward walks the
    products in reverse with those sums inside the kernels: each dense product's backward
    adds the sum's gradient to its in1 gradient (on the selected leading components) and
    accumulates its in2 gradient into the running gradient of the node features, which
    starts as the skip projection's input gradient and ends in the first map's epilogue."""

    @staticmethod
    def forward(ctx, node_feats, layer, *ws):
        comps = layer._selected_comps()
        width = comps * layer.in_features
        prods, prod = [], node_feats
        for step in range(layer.correlation):
            if step > 0:
                prod = layer.tensor_products[step - 1](prod, node_feats, ws[step - 1])
            if step < layer.correlation - 1:
                prod = layer.product_linears[step](prod)
                prods.append(prod)
        sel = (lambda p: p) if width == prods[0].shape[1] else (lambda p: p[:, :width].contiguous())
        acc = layer.skip_projection(node_feats, residual=sel(prods[0]))
        for p in prods[1:]:
            acc = acc + sel(p)
        out = layer.product_linears[layer.correlation - 1](prod, residual=acc)
        ctx.save_for_backward(node_feats, *prods, *ws)
        ctx.layer, ctx.comps, ctx.n_prods = layer, comps, len(prods)
        return out

    @staticmethod
    def backward(ctx, g):
        if torch.is_grad_enabled():
            raise RuntimeError("ProductLayer was evaluated inside first_order_only(); its backward cannot build a "
                               "graph for a second derivative")
        saved = ctx.saved_tensors
        x, prods, ws = saved[0], saved[1:1 + ctx.n_prods], saved[1 + ctx.n_prods:]
        layer, comps = ctx.layer, ctx.comps
        g = g.contiguous()
        if g.data_ptr() % 16:
            g = g.clone()
        _, precision = o3.utils.get_linear_triton_kernel_options(g.dtype)

        def input_grad(lin, rows):
            return ops._linear_input_grad(rows.contiguous(), lin.in_dim, list(lin.weight), lin.meta_lists, precision,
                                          lin.scale)

        g_t = input_grad(layer.product_linears[layer.correlation - 1], g)
        gx = input_grad(layer.skip_projection, g)  # the running gradient of the node features
        for k in range(layer.correlation - 1, 0, -1):
            g_prod, gx = ops.tp_dense_bwd_residual(layer.tensor_products[k - 1], g_t, prods[k - 1], x, ws[k - 1],
                                                   g, comps, gx, out_in2=gx)
            lin = layer.product_linears[k - 1]
            if k - 1 > 0:
                g_t = input_grad(lin, g_prod)
                continue
            in_offs, out_offs, _, m, fi, fo = lin.meta_lists
            if ops.linear_residual_layout_ok(lin.in_dim, lin.out_dim, m, fi, fo, in_offs, out_offs):
                gx = ops._linear_residual_impl(g_prod, list(lin.weight), lin.in_dim, lin.meta_lists, precision,
                                               lin.scale, gx, True, out=gx)
            else:
                gx = gx + input_grad(lin, g_prod)
        return (gx, None) + (None,) * len(ws)


class EnergyReadoutLayer(nn.Module):
    """MLP on the scalar channels of every layer (reference ``nn/layers.py:1021-1077``)."""

    def non_decayable_parameters(self) -> Iterator[nn.Parameter]:
        yield from iter_child_special_parameters(self, "non_decayable_parameters")

    def non_muon_parameters(self) -> Iterator[nn.Parameter]:
        # the last (single-output) layer goes to AdamW (reference nn/layers.py:1068-1070)
        yield from iter_child_special_parameters(self, "non_muon_parameters")
        yield self.readout_mlp[-1].weight

    def __init__(self, in_features: int, n_layers: int, hidden_readout: Optional[List[int]] = None):
        super().__init__()
        self.in_features = in_features
        self.n_layers = n_layers
        self.hidden_readout = [64, 64] if hidden_readout is None else list(hidden_readout)
        self.readout_mlp = _mlp([in_features * n_layers] + self.hidden_readout + [1])

    def forward(self, node_feats: List[torch.Tensor]) -> torch.Tensor:
        scalars = torch.cat([nf[:, :self.in_features] for nf in node_feats], dim=1)
        if scalars.shape[-1] != self.in_features * self.n_layers:
            raise RuntimeError(f"Incorrect last dimension for scalars. Expected: {self.in_features * self.n_layers}. "
                               f"Provided: {scalars.shape[-1]}.")
        return self.readout_mlp(scalars).squeeze(-1)


class ScaleShiftEnergyLayer(_NoSpecialParameters, nn.Module):
    """Per-element energy scale; shifts stored for calculators (reference ``nn/layers.py:1080-1138``)."""

    def __init__(self, n_elements: int):
        super().__init__()
        self.n_elements = n_elements
        self.register_buffer("shifts", torch.zeros(n_elements))
        self.register_buffer("scales", torch.ones(n_elements))

    def forward(self, node_output, atom_types):
        return self.scales[atom_types] * node_output
