"""Reference-compatible API (``import dst``) on top of dstraining_b200.

Module names and public symbols follow the reference package so that code
written against it runs unchanged; every symbol is the dstraining_b200 object
itself (not a copy), so patching e.g. ``dst.recompute._Recompute.forward``
affects the framework.
"""
