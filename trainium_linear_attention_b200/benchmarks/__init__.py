"""Module paths matching the reference's ``benchmarks`` package, so code that
imports the reference's host wrappers from there can switch by changing the
package prefix only."""
