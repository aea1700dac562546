"""Measured launch configurations for the CUDA folds -- only deviations from
`autotune.default_config` are listed, keyed by `(rows class, pow2 width bucket)`.

A machine without an entry uses the default. The b200 entry is empty until a measurement on a
B200 shows a candidate beating the default by more than `autotune.NOISE`.
"""
TABLES = {
    'b200': {
        'measured_on': 'NVIDIA B200 (no deviation from the default recorded yet)',
        'noise': 0.05,
        'table': {},
    },
}
