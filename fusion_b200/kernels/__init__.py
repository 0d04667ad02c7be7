"""Drop-in replacements for the reference's kernel modules (glm52/kernels/*.py).

Same module names, function names, argument order and destination-passing convention;
`cfg` dicts are accepted for signature compatibility (the Triton mapping knobs in them
do not apply to the sm_100a kernels; semantic keys such as `eps`, `scale`, `NORM_PROB`,
`ROUND_MID` are honoured).
"""
