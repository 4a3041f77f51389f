"""flyguy_b200: the connectome hop path of flyguy (obs -> input plug -> sparse hops -> output plug, its backward
pass and Adam) as hand-written sm_100a CUDA behind a C-ABI shared library, with flyguy's Python host API."""
__version__ = "0.1.0"
