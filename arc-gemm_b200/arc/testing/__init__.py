"""Test-side helpers: seeded data generators and device timers."""
