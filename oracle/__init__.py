"""CPU float64 oracle of GoTransformers' mixture-of-experts forward path.

Test infrastructure only (the checker of the parity tests, the smoke check and
the benchmark's CPU-baseline leg); the product never imports this package."""
