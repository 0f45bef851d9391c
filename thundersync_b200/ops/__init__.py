"""Native sm_100a ops with autograd, plus their exact CPU reference paths.

Every op here has one CUDA implementation (this package's extension, built
for sm_100a) and one CPU implementation in plain torch fp32 math that serves
as the test oracle and as the CPU execution path. There is no runtime
backend choice on CUDA: if the extension is missing on a CUDA device the op
raises.
"""
