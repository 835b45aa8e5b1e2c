"""Regenerate reference_abi_symbols.txt: every zeno_* function the reference's cffi binding
declares (python/zeno/_ffi.py cdef block of Lulzx/zeno), i.e. what its
tests/check_abi_contract.py requires the library to export.  Run where the reference
checkout is available:

    python tests/golden/make_reference_abi_list.py /path/to/zeno
"""
import re
import sys
from pathlib import Path

ref = Path(sys.argv[1])
text = (ref / "python" / "zeno" / "_ffi.py").read_text()
block = re.search(r'ffi\.cdef\(\s*"""(.*?)"""\s*\)', text, flags=re.S).group(1)
names = sorted(set(re.findall(r"\b(zeno_[A-Za-z0-9_]+)\s*\(", block)))
(Path(__file__).parent / "reference_abi_symbols.txt").write_text("\n".join(names) + "\n")
print(len(names), "symbols")
