"""Drop-in replacements for the hot-path modules of ``nanovllm.layers``.

Same class/function names, constructor arguments, parameters/buffers and
error messages as the reference modules; the math runs in the sm_100a kernels
of ``libnib_b200.so``.
"""
