// Compile-only stand-in for the Apple framework header that the reference's host
// files import.  Nothing the restated host generators use comes from it.
#pragma once
