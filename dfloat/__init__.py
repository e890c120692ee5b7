"""The ``dfloat`` import path of zeyuyang8/ecf8, served by ecf8_b200.

User code written against the reference package (dfloat/__init__.py:1,
dfloat/run/__init__.py:1-17) runs unchanged: ``from dfloat.run import
DFloatModel, _decode``, ``from dfloat import utils``, ``from dfloat.const
import get_fp8_pattern_dict``.  Every name resolves to the B200 engine in
``ecf8_b200``; nothing here implements anything of its own.
"""

__version__ = "0.0.0"
