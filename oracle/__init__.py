"""CPU oracle for the tree-verification path: test infrastructure, not product.

Only the test suite, the smoke check and the benchmark's CPU-baseline leg may
import this package.
"""
