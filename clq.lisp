;;;; clq.lisp -- CFFI binding of libclq (include/clq.h) for cl-inference's
;;;; packed kernels.  Copy to quant/clq.lisp and load it before
;;;; quant/packed.lisp; then rebind the kernel slots of quant/packed.lisp:156-158
;;;; and quant/q8-0.lisp:82 to the four functions below.  Each takes the
;;;; trivial-simd kernel's arguments (out x bytes M N K) and signals a Lisp
;;;; error when libclq returns a non-zero status.

(defpackage #:clq (:use #:cl)
  (:export #:q8-0-matmul! #:q4-0-matmul! #:q4-k-matmul! #:q6-k-matmul! #:forget))
(in-package #:clq)

(cffi:define-foreign-library libclq (t (:default "libclq")))
(cffi:use-foreign-library libclq)

(cffi:defcfun ("clq_last_error" %last-error) :int (buf :pointer) (len :size))
(cffi:defcfun ("clq_forget" %forget) :int (bytes :pointer) (nbytes :size))

(defun check (status)
  (unless (zerop status)
    (error "libclq: ~A"
           (cffi:with-foreign-pointer-as-string ((buf size) 1024) (%last-error buf size)))))

(defmacro with-storage-pointer ((var storage) &body body)
  "STORAGE is what cl-tensor hands the kernels: a trivial-simd vector view
(already a raw pointer, e.g. a mapped GGUF tensor) or a Lisp vector (pinned
for the call)."
  (let ((fn (gensym "BODY")) (s (gensym "STORAGE")) (p (gensym "POINTER")))
    `(let ((,s ,storage))
       (flet ((,fn (,var) ,@body))
         (if (simd:vector-view-p ,s)
             (,fn (simd:vector-view-pointer ,s))
             (cffi:with-pointer-to-vector-data (,p ,s) (,fn ,p)))))))

(defmacro define-kernel (name c-name)
  "NAME takes the trivial-simd kernel's arguments (out x bytes M N K)."
  (let ((foreign (intern (format nil "%~A" name))))
    `(progn
       (cffi:defcfun (,c-name ,foreign) :int
         (out :pointer) (x :pointer) (bytes :pointer) (m :int64) (n :int64) (k :int64))
       (defun ,name (out x bytes m n k)
         (with-storage-pointer (o out)
           (with-storage-pointer (xp x)
             (with-storage-pointer (b bytes)
               (check (,foreign o xp b m n k)))))
         out))))

(define-kernel q8-0-matmul! "clq_q8_0_matmul")
(define-kernel q4-0-matmul! "clq_q4_0_matmul")
(define-kernel q4-k-matmul! "clq_q4_k_matmul")
(define-kernel q6-k-matmul! "clq_q6_k_matmul")

(defun forget (pointer nbytes) (check (%forget pointer nbytes)))
