"""Measured launch configurations for the CUDA folds -- only deviations from
`autotune.default_config` are listed, keyed by `(rows class, pow2 width bucket)`.

Written by `python -m neptune_opt_b200.autotune --write` (autotune.measure_shapes on the
machine named in `measured_on`); a machine without an entry uses the default.
"""
TABLES = {
    'b200': {
        'measured_on': 'NVIDIA B200, logsumexp float32',
        'noise': 0.05,
        'table': {
        },
    },
}
