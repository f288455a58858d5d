"""Drop-in operator modules with the reference's submission surface.

Each module starts with the `# okc: problem=<name>` header of the reference's
`submission.py` files and exports `prepare(weights)` (untimed), `kernel_fn(data[, state])`
and `custom_kernel = kernel_fn`, taking the reference's `data` dictionaries
(muse_*/submission.py TypedDicts).  All compute runs in libokc_b200.so.
"""
