"""B200-native (sm_100a) FP8 dense-contraction path of macrogpt-jax: the FP8 mode of the
`Einsum` layer as used by `GMLP` and by the Q/K/V/O projections of `SoftmaxAttention`."""
