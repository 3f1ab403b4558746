"""The unmodified reference package, installed under baseline/_ref (test and bench comparator only)."""
