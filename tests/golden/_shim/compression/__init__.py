"""Fixture-generation shim: the reference imports `compression.zstd` (the
Python 3.14 stdlib module); this interpreter predates it, so make_golden.py
puts this package on sys.path to provide the four names the reference uses,
backed by the system libzstd.  Used only to run the reference here."""
