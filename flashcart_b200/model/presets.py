"""Architectures of the benchmark workloads: the 192-atom CPU reference run ("cfg0": 64 channels,
ranks <= 2) and the MD-scale inference step ("cfg3arch": 128 channels, ranks <= 3).

Flags of the reference's ``configs/default.yaml`` (layer norm, sigmoid gates, cosine
Chebyshev mapping, path-resolved products), fixed shifts, ``avg_neighbors`` set to
the measured mean degree of the structure.
"""

WATER_ARCHS = {
    "cfg0": dict(n_hidden_feats=64, l_max_hidden_feats=2, l_max_edge_attrs=2),
    "cfg3arch": dict(n_hidden_feats=128, l_max_hidden_feats=3, l_max_edge_attrs=3),
}
WATER_COMMON = dict(elements=["H", "O"], r_max=5.0, n_radial=8, n_interactions=2, correlation=3, layer_norm=True,
                    nonlinearity=True, gate_activation="sigmoid", radial_mapping="cosine",
                    path_reduced_product=False, fit_atomic_shifts=False, atomic_shifts=[0.0, 0.0])


def water_model_kwargs(name: str, avg_neighbors: float) -> dict:
    return dict(WATER_COMMON, **WATER_ARCHS[name], avg_neighbors=float(avg_neighbors))
