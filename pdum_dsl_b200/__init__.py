"""pdum_dsl_b200: a B200 (sm_100a) execution backend for pdum.dsl's fusion templates.

* ``kernels``   -- device-tensor entry points over the C ABI (include/pdb.h)
* ``tile``      -- ``compile_tile``: the reference lowering's call convention
* ``regions``   -- builders for the DSL regions the backend executes
"""

__version__ = "0.1.0"
