"""Drop-in mirror of the reference's ``kernels`` package.

Importing ``minimaxh3_b200.kernels.attention_router`` / ``.fp8_attention`` /
``.fp8_linear`` gives the same names and signatures as viragadel6/minimaxh3
``kernels/attention_router.py``, ``kernels/fp8_attention.py`` and
``kernels/fp8_linear.py``; the runtime can alias this package as ``kernels``.
``.lora.attach_lora_registry`` is the fused form of the reference's
``runtime/lora.py`` wrapper of the unquantised ``nn.Linear`` layers.
"""
