"""Drop-in counterparts of the reference's ``kernels`` package.

``pytorch_attention`` keeps the names and signatures of the reference's
kernels/pytorch_attention.py; ``chunked_attention`` and ``sliding_attention``
hold the host wrappers the reference keeps in its benchmark scripts.
"""
